// pkv_common.cuh — shared helpers of libpkv: status plumbing, dtype traits and
// the inline-PTX wrappers (mbarrier, TMA, ldmatrix, movmatrix, mma) the
// sm_100a kernels use.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/pkv.h"

namespace pkv {

// ---------------------------------------------------------------- host status
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define PKV_CUDA_RET(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::pkv::cuda_fail(_e, #expr); \
  } while (0)

inline int elem_size(int32_t dtype) {
  switch (dtype) {
    case PKV_F16: return 2;
    case PKV_BF16: return 2;
    case PKV_F32: return 4;
    case PKV_F64: return 8;
    default: return 0;
  }
}

// Validates a pool descriptor; returns PKV_OK or PKV_ERR_ARG with a message.
int check_pool(const pkv_pool* p);

inline int64_t row_bytes(const pkv_pool& p) {
  return (int64_t)p.n_kv_heads * p.head_dim * elem_size(p.dtype);
}
inline int64_t block_bytes(const pkv_pool& p) { return row_bytes(p) * p.block_size; }
inline int64_t slab_bytes(const pkv_pool& p) { return block_bytes(p) * p.num_blocks; }

int num_sms();  // SM count of the current device (cached per device)

// Programmatic dependent launch (PDL): the per-layer kernels of a step
// (append, decode) are launched so that the next one may be scheduled while
// the previous one drains; each waits (griddepcontrol.wait, a no-op when it was
// launched without the attribute) before it reads anything an earlier kernel
// wrote, so stream order still holds for every byte. PKV_PDL=0 turns it off.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Tensor map of a pool's permuted page view (dims D, token slot, KV head,
// layer*2+kv; one box = one whole [8 heads][16 tok][64] page of one layer's K
// or V), cached per (device, pool). pkv_attn.cu.
int pool_tmap(const pkv_pool& p, CUtensorMap* out);
// The same view with one KV head per box ([16 tok][64], 2 KiB for fp16).
int pool_tmap_head(const pkv_pool& p, CUtensorMap* out);

// Chunked-prefill / mixed-batch tensor-core attention (pkv_prefill.cu).
bool prefill_supported(const pkv_pool& p, int n_heads);
int prefill_tile_tokens(int n_heads, int n_kv_heads);
int64_t prefill_tiles_cap(int n_seqs, int64_t total_pages);
// Where the plan of a mixed batch lists its decode rows for the decode kernel
// (workspace regions; see pkv_attn.cu's workspace layout).
struct PrefillMixedPlan {
  int4* desc;          // [total_pages] page descriptors of the listed decode rows
  int32_t* counters;   // [n_seqs] split-K counters
  int32_t* rows;       // [n_seqs] q / out row of each listed sequence, -1 past the list
  int64_t* p_dec;      // pages listed
};
int prefill_plan(const pkv_pool& p, int n_heads, const pkv_batch& b, int2* tiles, int32_t* n_tiles,
                 int64_t tiles_cap, const PrefillMixedPlan* mixed, cudaStream_t s);
int prefill_attend(const pkv_pool& p, int layer, int n_heads, const void* q, void* out, float scale,
                   const pkv_batch& b, const int2* tiles, const int32_t* n_tiles, int64_t tiles_cap,
                   cudaStream_t s);
// The tcgen05 / TMEM variant (pkv_prefill_tc.cu); prefill_attend dispatches to it.
int prefill_tc_tile_tokens(int n_heads, int n_kv_heads);
int prefill_tc_attend(const pkv_pool& p, int layer, int n_heads, const void* q, void* out, float scale,
                      const pkv_batch& b, const int2* tiles, const int32_t* n_tiles, int64_t tiles_cap,
                      cudaStream_t s);

// ---------------------------------------------------------------- device side
// PDL: let the next kernel in the stream be scheduled now; wait until the
// kernels before this one completed and their writes are visible.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void flag(int32_t* st, int32_t bits) {
  if (st) atomicOr(st, bits);
}

// Exclusive prefix sum of v over the CTA (every thread calls it); *total gets the sum.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_sum, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += u;
  }
  __syncthreads();
  if (lane == 31) warp_sum[w] = incl;
  __syncthreads();
  if (w == 0) {
    int x = lane < nw ? warp_sum[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += u;
    }
    warp_sum[lane] = x;
  }
  __syncthreads();
  *total = warp_sum[nw - 1];
  return (w ? warp_sum[w - 1] : 0) + incl - v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// mbarrier ------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// One probe of phase `parity` (the hardware may suspend the thread for a
// system-dependent time while the phase is incomplete); true once it completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Waits at most ~1 s of wall time; on giving up ORs PKV_DEV_WAIT_TIMEOUT and
// returns false so the caller can unwind instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* st) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < 1000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  flag(st, PKV_DEV_WAIT_TIMEOUT);
  return false;
}

// 2^x on the SFU (PTX ex2.approx, flush-to-zero): inputs here are <= 0 and
// outputs are probabilities, where its relative error (< 2^-22) is irrelevant.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// As mbar_wait_bounded, for waiters off the critical path (the decode
// kernel's producer and merge warps): sleeps `ns` between probes so a waiting
// warp does not take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_wait_bounded_sleepy(uint64_t* bar, uint32_t parity, int32_t* st,
                                                         unsigned ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < 1000000000ull) {
    __nanosleep(ns);
    if (mbar_try_wait(bar, parity)) return true;
  }
  flag(st, PKV_DEV_WAIT_TIMEOUT);
  return false;
}

// TMA -----------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 4-D tiled TMA load into this CTA's own shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                           int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// Prefetch of a 4-D tile into L2 (no shared memory written, no completion to
// wait for): warms the cache for a later tma_load_4d of the same tile.
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// warp-level tensor-core helpers (fp16 / bf16 operands, fp32 accumulate) ----
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct MmaOp;
template <>
struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <>
struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// scalar conversions for the generic kernels
template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }

// Rotary embedding of one pair (a, b) = (x[i], x[i + D/2]) by the angle whose
// cosine is c and sine s: a' = a*c - b*s, b' = a*s + b*c, with every product
// rounded to fp32 before the difference / sum (no fused multiply-add), which is
// how the fp32 elementwise evaluation of that formula rounds.
__device__ __forceinline__ void rope_pair(float& a, float& b, float c, float s) {
  const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  const float rb = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  a = ra;
  b = rb;
}

// two 16-bit values packed in a word (lower index in the low half) <-> floats
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace pkv
