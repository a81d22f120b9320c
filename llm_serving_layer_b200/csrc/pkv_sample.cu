// pkv_sample.cu — greedy sampling on the device.
//
// The reference scheduler samples with torch.argmax(logits, dim=-1).tolist()
// after every forward pass (serving/scheduler/scheduler.py:756-757): the host
// waits for the step it just issued. Here the argmax runs as one launch that
// also writes each row's token into a device token table (the next step's
// input is assembled from it on the device), and optionally into a compact
// [n_rows] array the host reads back asynchronously, one step later.
//
// Semantics are torch.argmax's: the first index of the row maximum; a NaN
// counts as larger than every number (the first NaN wins); -0 and +0 are equal.
// Each element becomes a 32-bit key whose unsigned order is that order (IEEE
// bits with the sign folded: ~b for negatives, b | 2^31 otherwise; NaN ->
// 0xffffffff), and (key << 32) | ~index orders candidates so that the larger
// value, then the smaller index, wins: the row's token is the maximum of these
// 64-bit words, whatever order they are combined in.
//
// HBM-bound (one pass over the logits: 2 or 4 B per element). A CTA of 512
// threads streams its share of a row with 16-byte loads, four in flight per
// thread; per 16-byte vector only its maximum is compared with the thread's
// best (the vector is searched for the index only when that beats it). Small
// batches (fewer rows than two CTAs per SM) split each row over a thread-block
// cluster of 2-8 CTAs; the cluster combines its partial maxima through
// distributed shared memory, so no global scratch and no atomics.
#include <cooperative_groups.h>

#include <algorithm>

#include "pkv_common.cuh"

namespace cg = cooperative_groups;

namespace pkv {
namespace {

constexpr int SG_THREADS = 512;
constexpr int SG_UNROLL = 4;

__device__ __forceinline__ uint32_t order_key(float v) {
  if (v != v) return 0xFFFFFFFFu;
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0u;  // -0 == +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <typename T>
struct Vec;
// Vec<T>::vmax: the largest of a vector's elements, a NaN if it holds one (the
// order_key order up to the sign of zero, which order_key folds).
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static float vmax(const uint4& u) {
    const float a = __uint_as_float(u.x), b = __uint_as_float(u.y), c = __uint_as_float(u.z),
                d = __uint_as_float(u.w);
    const float m = fmaxf(fmaxf(a, b), fmaxf(c, d));  // fmaxf drops NaNs: put one back
    return (a != a || b != b || c != c || d != d) ? __uint_as_float(0x7fffffffu) : m;
  }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = unpack2<__half>(w[i]);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ __forceinline__ static float vmax(const uint4& u) {
    const __half2 m = __hmax2_nan(__hmax2_nan(*reinterpret_cast<const __half2*>(&u.x),
                                              *reinterpret_cast<const __half2*>(&u.y)),
                                  __hmax2_nan(*reinterpret_cast<const __half2*>(&u.z),
                                              *reinterpret_cast<const __half2*>(&u.w)));
    return __half2float(__hmax_nan(__low2half(m), __high2half(m)));
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = unpack2<__nv_bfloat16>(w[i]);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ __forceinline__ static float vmax(const uint4& u) {
    const __nv_bfloat162 m = __hmax2_nan(__hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&u.x),
                                                     *reinterpret_cast<const __nv_bfloat162*>(&u.y)),
                                         __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&u.z),
                                                     *reinterpret_cast<const __nv_bfloat162*>(&u.w)));
    return __bfloat162float(__hmax_nan(__low2bfloat16(m), __high2bfloat16(m)));
  }
};

__device__ __forceinline__ uint64_t pack_best(uint32_t key, uint32_t idx) {
  return (uint64_t(key) << 32) | uint64_t(~idx);
}

// A vector of elements [base, base + N): its maximum's key is compared with
// the thread's best; only a vector that beats it is searched for the first
// element holding that key (rare once a row's large values have been seen).
template <typename T>
__device__ __forceinline__ void take_vec(const uint4& u, uint32_t base, uint32_t& best_key, uint32_t& best_idx) {
  constexpr int N = Vec<T>::N;
  const uint32_t vk = order_key(Vec<T>::vmax(u));
  if (vk > best_key) {
    float f[N];
    Vec<T>::unpack(u, f);
    int first = N - 1;
#pragma unroll
    for (int e = N - 1; e >= 0; --e)
      if (order_key(f[e]) == vk) first = e;
    best_key = vk;
    best_idx = base + first;
  }
}

// One CTA's share of a row: [lo, hi) element indices. Threads visit their
// indices in increasing order, so a strict comparison keeps each thread's
// first maximum; the 64-bit combine then keeps the smallest index overall.
template <typename T, bool VEC>
__device__ __forceinline__ uint64_t scan_share(const T* __restrict__ row, int64_t lo, int64_t hi) {
  uint32_t best_key = 0, best_idx = 0;
  int64_t i = lo;
  if (VEC) {
    constexpr int N = Vec<T>::N;
    // lo is a multiple of N (the host splits rows on vector boundaries)
    const int64_t nvec = (hi - lo) / N;
    const uint4* v = reinterpret_cast<const uint4*>(row + lo);
    int64_t k = threadIdx.x;
    for (; k + int64_t(SG_UNROLL - 1) * SG_THREADS < nvec; k += int64_t(SG_UNROLL) * SG_THREADS) {
      uint4 u[SG_UNROLL];
#pragma unroll
      for (int j = 0; j < SG_UNROLL; ++j) u[j] = __ldcs(v + k + int64_t(j) * SG_THREADS);
#pragma unroll
      for (int j = 0; j < SG_UNROLL; ++j)
        take_vec<T>(u[j], uint32_t(lo + (k + int64_t(j) * SG_THREADS) * N), best_key, best_idx);
    }
    for (; k < nvec; k += SG_THREADS) take_vec<T>(__ldcs(v + k), uint32_t(lo + k * N), best_key, best_idx);
    i = lo + nvec * N;
  }
  for (int64_t e = i + threadIdx.x; e < hi; e += SG_THREADS) {
    const uint32_t key = order_key(to_f<T>(row[e]));
    if (key > best_key) {
      best_key = key;
      best_idx = uint32_t(e);
    }
  }
  uint64_t best = best_key ? pack_best(best_key, best_idx) : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ uint64_t warp_best[SG_THREADS / 32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) warp_best[w] = best;
  __syncthreads();
  if (w == 0) {
    best = l < SG_THREADS / 32 ? warp_best[l] : 0ull;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  }
  return best;  // valid in warp 0
}

struct SampleArgs {
  const void* logits;
  int64_t n_rows;
  int64_t vocab;
  int64_t row_stride;  // elements
  int64_t share;       // elements per cluster rank (a multiple of the vector width)
  const int32_t* rows;
  int64_t* tokens;
  int64_t tokens_len;
  int64_t* sampled;
  int32_t* st;
};

// grid.x = n_rows * cluster size; cluster rank c scans [c*share, min((c+1)*share, vocab)).
template <typename T, bool VEC>
__global__ void __launch_bounds__(SG_THREADS) sample_greedy_kernel(SampleArgs a) {
  pdl_trigger();
  pdl_wait();  // the logits come from the GEMM just before
  const cg::cluster_group cluster = cg::this_cluster();
  const unsigned cs = cluster.num_blocks();
  const unsigned rank = cluster.block_rank();
  const int64_t r = int64_t(blockIdx.x) / cs;
  const T* row = static_cast<const T*>(a.logits) + r * a.row_stride;
  const int64_t lo = std::min<int64_t>(int64_t(rank) * a.share, a.vocab);
  const int64_t hi = std::min<int64_t>(lo + a.share, a.vocab);
  __shared__ uint64_t cta_best;
  const uint64_t best = scan_share<T, VEC>(row, lo, hi);
  if (threadIdx.x == 0) cta_best = best;
  if (cs > 1) cluster.sync();  // every rank's cta_best written
  else __syncthreads();
  if (rank == 0 && threadIdx.x == 0) {
    uint64_t b = cta_best;
    for (unsigned c = 1; c < cs; ++c) b = max(b, *cluster.map_shared_rank(&cta_best, c));
    const int64_t tok = int64_t(~uint32_t(b & 0xFFFFFFFFull));
    if (a.sampled) a.sampled[r] = tok;
    if (a.rows) {
      const int32_t dst = a.rows[r];
      if (dst >= 0) {
        if (dst < a.tokens_len) a.tokens[dst] = tok;
        else flag(a.st, PKV_DEV_SLOT_OOB);
      }
    } else if (a.tokens) {
      a.tokens[r] = tok;
    }
  }
  if (cs > 1) cluster.sync();  // rank 0 has read every peer's shared memory
}

template <typename T, bool VEC>
int launch_sample(const SampleArgs& a, int cs, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(a.n_rows * cs));
  cfg.blockDim = dim3(SG_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(cs);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  PKV_CUDA_RET(cudaLaunchKernelEx(&cfg, sample_greedy_kernel<T, VEC>, a));
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

template <typename T>
int sample_typed(SampleArgs a, cudaStream_t s) {
  constexpr int N = Vec<T>::N;
  const bool vec = (reinterpret_cast<uintptr_t>(a.logits) % 16 == 0) && (a.row_stride % N == 0);
  // cluster size: enough CTAs for two per SM, each with at least a few
  // vectors per thread; rows are split on vector boundaries
  const int64_t want_ctas = 2 * int64_t(num_sms());
  int cs = 1;
  while (cs < 8 && a.n_rows * cs < want_ctas && a.vocab / (2 * cs) >= int64_t(SG_THREADS) * N * 2) cs *= 2;
  int64_t share = (a.vocab + cs - 1) / cs;
  share = (share + N - 1) / N * N;
  a.share = share;
  if (a.n_rows * cs > 0x7fffffffLL) return fail(PKV_ERR_ARG, "too many logits rows for one launch");
  return vec ? launch_sample<T, true>(a, cs, s) : launch_sample<T, false>(a, cs, s);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_sample_greedy(int32_t dtype, const void* logits, int64_t n_rows, int64_t vocab,
                                 int64_t row_stride, const int32_t* rows, int64_t* tokens, int64_t tokens_len,
                                 int64_t* sampled, int32_t* dev_status, void* stream) {
  if (dtype != PKV_F16 && dtype != PKV_BF16 && dtype != PKV_F32)
    return fail(PKV_ERR_UNSUPPORTED, "pkv_sample_greedy takes fp16, bf16 or fp32 logits");
  if (n_rows < 0) return fail(PKV_ERR_ARG, "n_rows must be >= 0");
  if (vocab <= 0 || vocab >= (int64_t(1) << 31)) return fail(PKV_ERR_ARG, "vocab must be in [1, 2^31)");
  if (row_stride < vocab) return fail(PKV_ERR_ARG, "row_stride must be >= vocab");
  if (!tokens && !sampled) return fail(PKV_ERR_ARG, "give tokens, sampled or both");
  if (tokens_len < 0) return fail(PKV_ERR_ARG, "tokens_len must be >= 0");
  if (tokens && !rows && tokens_len < n_rows)
    return fail(PKV_ERR_ARG, "without rows, tokens must hold n_rows entries");
  if (rows && !tokens) return fail(PKV_ERR_ARG, "rows given without a tokens table");
  if (n_rows == 0) return PKV_OK;
  if (!logits) return fail(PKV_ERR_ARG, "logits must be non-NULL");
  SampleArgs a;
  a.logits = logits;
  a.n_rows = n_rows;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.share = 0;
  a.rows = rows;
  a.tokens = tokens;
  a.tokens_len = tokens_len;
  a.sampled = sampled;
  a.st = dev_status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PKV_F16: return sample_typed<__half>(a, s);
    case PKV_BF16: return sample_typed<__nv_bfloat16>(a, s);
    default: return sample_typed<float>(a, s);
  }
}
