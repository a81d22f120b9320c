// pkv_copy.cu — the byte-moving half of the hot path: KV-append scatter,
// batched copy-on-write block copies, swap gather/scatter kernels and the
// asynchronous swap engine (copy-engine transfers on a private stream).
//
// All of these are HBM-bound byte copies: the kernels move 16-byte vectors
// with coalesced loads and stores and never reshape the work into GEMMs.
#include <deque>
#include <map>
#include <vector>
#include <string>

#include "pkv_common.cuh"

namespace pkv {

namespace {

// Widest vector type dividing every byte count and address involved.
inline int vec_width(int64_t bytes, std::initializer_list<const void*> ptrs) {
  int w = 16;
  while (w > 1) {
    bool ok = (bytes % w) == 0;
    for (const void* p : ptrs) ok = ok && ((reinterpret_cast<uintptr_t>(p) % w) == 0);
    if (ok) break;
    w >>= 1;
  }
  return w;
}

template <int W>
struct Vec;
template <>
struct Vec<16> { using T = uint4; };
template <>
struct Vec<8> { using T = uint2; };
template <>
struct Vec<4> { using T = uint32_t; };
template <>
struct Vec<2> { using T = uint16_t; };
template <>
struct Vec<1> { using T = uint8_t; };

// ------------------------------------------------------------------ append
// One warp per (token, K|V) row; the row (n_kv_heads * head_dim elements) is
// contiguous both in the input and at its slot in the pool.
template <int W>
__global__ void __launch_bounds__(256) append_kernel(char* __restrict__ k_slab,
                                                     char* __restrict__ v_slab,
                                                     const char* __restrict__ k,
                                                     const char* __restrict__ v,
                                                     const int32_t* __restrict__ slots,
                                                     int64_t n_tokens, int64_t n_slots,
                                                     int64_t row_bytes, int32_t* st) {
  using T = typename Vec<W>::T;
  pdl_trigger();
  pdl_wait();  // k, v and slot_mapping may come from the kernels just before
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= 2 * n_tokens) return;
  const int64_t tok = warp >> 1;
  const int kv = int(warp & 1);
  // The row's data does not depend on its slot: both loads are issued before
  // either is used, so the kernel pays one memory round trip, not two in a row.
  const int64_t slot = slots[tok];
  const T* src = reinterpret_cast<const T*>((kv ? v : k) + tok * row_bytes);
  const int64_t n = row_bytes / W;
  constexpr int U = 4;  // vectors per lane in flight
  for (int64_t i0 = lane; i0 < n; i0 += 32 * U) {
    T buf[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + 32 * u < n) buf[u] = __ldg(src + i0 + 32 * u);
    if (slot < 0 || slot >= n_slots) {
      if (lane == 0 && kv == 0) flag(st, PKV_DEV_SLOT_OOB);
      return;
    }
    T* dst = reinterpret_cast<T*>((kv ? v_slab : k_slab) + slot * row_bytes);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + 32 * u < n) dst[i0 + 32 * u] = buf[u];
  }
}

// ------------------------------------------------------------------ copy blocks
// blockIdx.x = pair * (2L) + (2*layer + kv); the CTA copies one block_bytes segment.
template <int W>
__global__ void __launch_bounds__(256) copy_blocks_kernel(char* __restrict__ base,
                                                          const int32_t* __restrict__ src,
                                                          const int32_t* __restrict__ dst,
                                                          int64_t n_pairs, int32_t n_slabs,
                                                          int64_t num_blocks, int64_t block_bytes,
                                                          int64_t slab_bytes, int32_t* st) {
  using T = typename Vec<W>::T;
  const int64_t seg = blockIdx.x;
  const int64_t pair = seg / n_slabs;
  const int slab = int(seg % n_slabs);
  if (pair >= n_pairs) return;
  const int64_t s = src[pair], d = dst[pair];
  if (s < 0 || s >= num_blocks || d < 0 || d >= num_blocks) {
    if (threadIdx.x == 0 && slab == 0) flag(st, PKV_DEV_SLOT_OOB);
    return;
  }
  if (s == d) return;
  const T* from = reinterpret_cast<const T*>(base + slab * slab_bytes + s * block_bytes);
  T* to = reinterpret_cast<T*>(base + slab * slab_bytes + d * block_bytes);
  const int64_t n = block_bytes / W;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) to[i] = from[i];
}

// One pair given by value (the reference's copy_block(src, dst) signature):
// blockIdx.x = 2*layer + kv.
template <int W>
__global__ void __launch_bounds__(256) copy_one_kernel(char* __restrict__ base, int64_t s,
                                                       int64_t d, int64_t block_bytes,
                                                       int64_t slab_bytes) {
  using T = typename Vec<W>::T;
  const int64_t slab = blockIdx.x;
  const T* from = reinterpret_cast<const T*>(base + slab * slab_bytes + s * block_bytes);
  T* to = reinterpret_cast<T*>(base + slab * slab_bytes + d * block_bytes);
  const int64_t n = block_bytes / W;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) to[i] = from[i];
}

// ------------------------------------------------------------------ swap
// Segment j of a swapped sequence (j in [0, 2*L*nb)): kv = j / (L*nb),
// layer = (j / nb) % L, block i = j % nb; host/staging offset j * block_bytes.
// GATHER: pool -> staging[(j - j0) * bb];  SCATTER: staging -> pool.
template <int W, bool GATHER>
__global__ void __launch_bounds__(256) swap_kernel(char* __restrict__ base,
                                                   const int32_t* __restrict__ ids, int64_t nb,
                                                   int32_t num_layers, int64_t num_blocks,
                                                   int64_t block_bytes, int64_t slab_bytes,
                                                   char* __restrict__ staging, int64_t j0,
                                                   int64_t count, int32_t* st) {
  using T = typename Vec<W>::T;
  const int64_t jj = blockIdx.x;
  if (jj >= count) return;
  const int64_t j = j0 + jj;
  const int64_t per_kv = int64_t(num_layers) * nb;
  const int kv = int(j / per_kv);
  const int64_t layer = (j / nb) % num_layers;
  const int64_t i = j % nb;
  const int64_t b = ids[i];
  if (b < 0 || b >= num_blocks) {
    if (threadIdx.x == 0) flag(st, PKV_DEV_SLOT_OOB);
    return;
  }
  char* pool_seg = base + (2 * layer + kv) * slab_bytes + b * block_bytes;
  char* stage_seg = staging + jj * block_bytes;
  const T* from = reinterpret_cast<const T*>(GATHER ? pool_seg : stage_seg);
  T* to = reinterpret_cast<T*>(GATHER ? stage_seg : pool_seg);
  const int64_t n = block_bytes / W;
  for (int64_t t = threadIdx.x; t < n; t += blockDim.x) to[t] = from[t];
}

template <bool GATHER>
int launch_swap(const pkv_pool& p, const int32_t* ids, int64_t nb, char* staging, int64_t j0,
                int64_t count, int32_t* st, cudaStream_t s) {
  if (count <= 0) return PKV_OK;
  const int64_t bb = block_bytes(p), sb = slab_bytes(p);
  const int w = vec_width(bb, {p.base, staging});
  const dim3 grid((unsigned)count), block(256);
  char* base = static_cast<char*>(p.base);
#define PKV_SWAP_CASE(WW)                                                                     \
  case WW:                                                                                    \
    swap_kernel<WW, GATHER><<<grid, block, 0, s>>>(base, ids, nb, p.num_layers, p.num_blocks, \
                                                   bb, sb, staging, j0, count, st);           \
    break;
  switch (w) {
    PKV_SWAP_CASE(16)
    PKV_SWAP_CASE(8)
    PKV_SWAP_CASE(4)
    PKV_SWAP_CASE(2)
    PKV_SWAP_CASE(1)
  }
#undef PKV_SWAP_CASE
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_append_kv(const pkv_pool* pool, int32_t layer, const void* k, const void* v,
                             const int32_t* slot_mapping, int64_t n_tokens, int32_t* dev_status,
                             void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (layer < 0 || layer >= p.num_layers)
    return fail(PKV_ERR_ARG, "layer_idx " + std::to_string(layer) + " out of range [0, " +
                                 std::to_string(p.num_layers) + ")");
  if (n_tokens < 0) return fail(PKV_ERR_ARG, "n_tokens must be >= 0");
  if (n_tokens == 0) return PKV_OK;
  if (!k || !v || !slot_mapping) return fail(PKV_ERR_ARG, "k, v and slot_mapping must be non-NULL");
  const int64_t rb = row_bytes(p), sb = slab_bytes(p);
  char* k_slab = static_cast<char*>(p.base) + (2 * int64_t(layer)) * sb;
  char* v_slab = k_slab + sb;
  const int w = vec_width(rb, {p.base, k, v});
  const int64_t threads = 2 * n_tokens * 32;
  const dim3 block(256), grid((unsigned)((threads + 255) / 256));
  const int64_t n_slots = p.num_blocks * p.block_size;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const char* kk = static_cast<const char*>(k);
  const char* vv = static_cast<const char*>(v);
#define PKV_APPEND_CASE(WW)                                                                       \
  case WW:                                                                                        \
    PKV_CUDA_RET(launch_kernel(append_kernel<WW>, grid, block, 0, s, true, k_slab, v_slab, kk, vv, \
                               slot_mapping, n_tokens, n_slots, rb, dev_status));                 \
    break;
  switch (w) {
    PKV_APPEND_CASE(16)
    PKV_APPEND_CASE(8)
    PKV_APPEND_CASE(4)
    PKV_APPEND_CASE(2)
    PKV_APPEND_CASE(1)
  }
#undef PKV_APPEND_CASE
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

extern "C" int pkv_copy_blocks(const pkv_pool* pool, const int32_t* src, const int32_t* dst,
                               int64_t n_pairs, int32_t* dev_status, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (n_pairs < 0) return fail(PKV_ERR_ARG, "n_pairs must be >= 0");
  if (n_pairs == 0) return PKV_OK;
  if (!src || !dst) return fail(PKV_ERR_ARG, "src and dst must be non-NULL");
  const int64_t bb = block_bytes(p), sb = slab_bytes(p);
  const int32_t n_slabs = 2 * p.num_layers;
  const int64_t n_ctas = n_pairs * n_slabs;
  if (n_ctas >= (int64_t(1) << 31)) return fail(PKV_ERR_ARG, "too many pairs for one launch");
  const int w = vec_width(bb, {p.base});
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(p.base);
#define PKV_COPY_CASE(WW)                                                                  \
  case WW:                                                                                 \
    copy_blocks_kernel<WW><<<(unsigned)n_ctas, 256, 0, s>>>(base, src, dst, n_pairs, n_slabs, \
                                                            p.num_blocks, bb, sb, dev_status); \
    break;
  switch (w) {
    PKV_COPY_CASE(16)
    PKV_COPY_CASE(8)
    PKV_COPY_CASE(4)
    PKV_COPY_CASE(2)
    PKV_COPY_CASE(1)
  }
#undef PKV_COPY_CASE
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

extern "C" int pkv_copy_block(const pkv_pool* pool, int64_t src, int64_t dst, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (src < 0 || src >= p.num_blocks || dst < 0 || dst >= p.num_blocks)
    return fail(PKV_ERR_ARG, "copy_block(" + std::to_string(src) + " -> " + std::to_string(dst) +
                                 ") outside [0, " + std::to_string(p.num_blocks) + ")");
  if (src == dst) return PKV_OK;
  const int64_t bb = block_bytes(p), sb = slab_bytes(p);
  const int w = vec_width(bb, {p.base});
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(p.base);
  const unsigned n_slabs = unsigned(2 * p.num_layers);
#define PKV_COPY1_CASE(WW)                                                   \
  case WW:                                                                   \
    copy_one_kernel<WW><<<n_slabs, 256, 0, s>>>(base, src, dst, bb, sb);     \
    break;
  switch (w) {
    PKV_COPY1_CASE(16)
    PKV_COPY1_CASE(8)
    PKV_COPY1_CASE(4)
    PKV_COPY1_CASE(2)
    PKV_COPY1_CASE(1)
  }
#undef PKV_COPY1_CASE
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

extern "C" int pkv_swap_gather(const pkv_pool* pool, const int32_t* block_ids, int64_t nb,
                               void* staging, int32_t* dev_status, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  if (nb < 0) return fail(PKV_ERR_ARG, "nb must be >= 0");
  if (nb == 0) return PKV_OK;
  if (!block_ids || !staging) return fail(PKV_ERR_ARG, "block_ids and staging must be non-NULL");
  const int64_t segs = 2 * int64_t(pool->num_layers) * nb;
  if (segs >= (int64_t(1) << 31)) return fail(PKV_ERR_ARG, "swap too large for one launch");
  return launch_swap<true>(*pool, block_ids, nb, static_cast<char*>(staging), 0, segs, dev_status,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int pkv_swap_scatter(const pkv_pool* pool, const int32_t* block_ids, int64_t nb,
                                const void* staging, int32_t* dev_status, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  if (nb < 0) return fail(PKV_ERR_ARG, "nb must be >= 0");
  if (nb == 0) return PKV_OK;
  if (!block_ids || !staging) return fail(PKV_ERR_ARG, "block_ids and staging must be non-NULL");
  const int64_t segs = 2 * int64_t(pool->num_layers) * nb;
  if (segs >= (int64_t(1) << 31)) return fail(PKV_ERR_ARG, "swap too large for one launch");
  return launch_swap<false>(*pool, block_ids, nb, const_cast<char*>(static_cast<const char*>(staging)),
                            0, segs, dev_status, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ swap engine

// Staging is a ring: each chunk of a transfer takes the next contiguous region
// (wrapping to the start when the tail is too short) and waits, on the stream
// that writes it, only for the earlier uses it overlaps. A use ends at an event
// recorded after the last operation that reads or writes the region (the D2H
// copy of a swap-out, the scatter kernel of a swap-in); ended uses are pruned
// by querying their events. So transfers smaller than the staging area do not
// wait for one another, and the gather of a swap-out (which the compute stream
// waits for) waits for a host copy only once the staging area is full.
struct StageUse {
  size_t off, len;
  cudaEvent_t done;
};

struct pkv_swapper {
  int device = 0;
  char* staging = nullptr;
  size_t staging_bytes = 0;
  size_t chunk_bytes = 0;          // largest region one chunk takes (half the ring)
  size_t head = 0;                 // next free offset of the ring
  std::deque<StageUse> uses;       // regions in use, oldest first
  std::vector<cudaEvent_t> spare;  // events of ended uses, for reuse
  cudaStream_t kstream = nullptr;  // gather / scatter kernels
  cudaStream_t cstream = nullptr;  // copy-engine transfers
  cudaEvent_t ready = nullptr;     // a chunk's first stage done (gathered, resp. copied in)
  cudaEvent_t ev_start = nullptr, ev_kdone = nullptr;
  uint64_t next_ticket = 1;
  std::map<uint64_t, cudaEvent_t> tickets;
};

namespace pkv {
namespace {

int check_swapper(pkv_swapper* sw) {
  if (!sw) return fail(PKV_ERR_ARG, "swapper is NULL");
  int dev = -1;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  if (dev != sw->device)
    return fail(PKV_ERR_ARG, "swapper used on device " + std::to_string(dev) + " but created on " +
                                 std::to_string(sw->device));
  return PKV_OK;
}

// A region of `len` bytes (<= chunk_bytes) for a chunk written on `writer`:
// `writer` waits for every earlier use the region overlaps.
int stage_alloc(pkv_swapper* sw, size_t len, cudaStream_t writer, size_t* off) {
  while (!sw->uses.empty()) {  // prune the uses that ended
    const cudaError_t q = cudaEventQuery(sw->uses.front().done);
    if (q == cudaErrorNotReady) break;
    if (q != cudaSuccess) return cuda_fail(q, "cudaEventQuery");
    sw->spare.push_back(sw->uses.front().done);
    sw->uses.pop_front();
  }
  size_t o = sw->head;
  if (o + len > sw->staging_bytes) o = 0;
  for (const StageUse& u : sw->uses)
    if (u.off < o + len && o < u.off + u.len) PKV_CUDA_RET(cudaStreamWaitEvent(writer, u.done, 0));
  sw->head = o + len;
  *off = o;
  return PKV_OK;
}

// The region [off, off + len) is in use until the work queued on `last` so far.
int stage_release(pkv_swapper* sw, size_t off, size_t len, cudaStream_t last) {
  cudaEvent_t e;
  if (!sw->spare.empty()) {
    e = sw->spare.back();
    sw->spare.pop_back();
  } else {
    PKV_CUDA_RET(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  PKV_CUDA_RET(cudaEventRecord(e, last));
  sw->uses.push_back({off, len, e});
  return PKV_OK;
}

int new_ticket(pkv_swapper* sw, cudaStream_t s, uint64_t* ticket) {
  cudaEvent_t e;
  PKV_CUDA_RET(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  PKV_CUDA_RET(cudaEventRecord(e, s));
  const uint64_t t = sw->next_ticket++;
  sw->tickets[t] = e;
  if (ticket) *ticket = t;
  return PKV_OK;
}

// Host byte address of segment j in the (K buffer, V buffer) pair.
inline char* host_seg(char* hk, char* hv, int64_t j, int64_t per_kv, int64_t bb) {
  return j < per_kv ? hk + j * bb : hv + (j - per_kv) * bb;
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_swapper_create(void* staging, size_t staging_bytes, pkv_swapper** out) {
  if (!out) return fail(PKV_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (!staging || staging_bytes < 2 * 16) return fail(PKV_ERR_ARG, "staging buffer too small");
  if (reinterpret_cast<uintptr_t>(staging) % 16) return fail(PKV_ERR_ARG, "staging must be 16-byte aligned");
  pkv_swapper* sw = new pkv_swapper();
  sw->staging = static_cast<char*>(staging);
  sw->staging_bytes = staging_bytes & ~size_t(15);
  sw->chunk_bytes = (staging_bytes / 2) & ~size_t(15);
  cudaError_t e = cudaGetDevice(&sw->device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&sw->kstream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&sw->cstream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sw->ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sw->ev_start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sw->ev_kdone, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    pkv_swapper_destroy(sw);
    return cuda_fail(e, "pkv_swapper_create");
  }
  *out = sw;
  return PKV_OK;
}

extern "C" int pkv_swapper_destroy(pkv_swapper* sw) {
  if (!sw) return PKV_OK;
  if (sw->kstream) cudaStreamSynchronize(sw->kstream);
  if (sw->cstream) cudaStreamSynchronize(sw->cstream);
  for (auto& kv : sw->tickets) cudaEventDestroy(kv.second);
  for (auto& u : sw->uses) cudaEventDestroy(u.done);
  for (auto ev : sw->spare) cudaEventDestroy(ev);
  if (sw->ready) cudaEventDestroy(sw->ready);
  if (sw->ev_start) cudaEventDestroy(sw->ev_start);
  if (sw->ev_kdone) cudaEventDestroy(sw->ev_kdone);
  if (sw->kstream) cudaStreamDestroy(sw->kstream);
  if (sw->cstream) cudaStreamDestroy(sw->cstream);
  delete sw;
  return PKV_OK;
}

extern "C" int pkv_swap_out(pkv_swapper* sw, const pkv_pool* pool, const int32_t* block_ids,
                            int64_t nb, void* host_k, void* host_v, void* compute_stream,
                            int32_t* dev_status, uint64_t* ticket) {
  if (int rc = check_swapper(sw)) return rc;
  if (int rc = check_pool(pool)) return rc;
  if (nb < 0) return fail(PKV_ERR_ARG, "nb must be >= 0");
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  if (nb == 0) return new_ticket(sw, sw->cstream, ticket);
  if (!block_ids || !host_k || !host_v) return fail(PKV_ERR_ARG, "block_ids and host buffers must be non-NULL");
  const pkv_pool& p = *pool;
  const int64_t bb = block_bytes(p);
  const int64_t chunk = int64_t(sw->chunk_bytes) / bb;
  if (chunk < 1) return fail(PKV_ERR_ARG, "staging half smaller than one block");
  const int64_t per_kv = int64_t(p.num_layers) * nb, segs = 2 * per_kv;
  char* hk = static_cast<char*>(host_k);
  char* hv = static_cast<char*>(host_v);

  // everything already queued on the compute stream (appends) happens first
  PKV_CUDA_RET(cudaEventRecord(sw->ev_start, cs));
  PKV_CUDA_RET(cudaStreamWaitEvent(sw->kstream, sw->ev_start, 0));
  for (int64_t j0 = 0; j0 < segs; j0 += chunk) {
    const int64_t cnt = std::min(chunk, segs - j0);
    size_t off = 0;
    if (int rc = stage_alloc(sw, size_t(cnt * bb), sw->kstream, &off)) return rc;
    char* stage = sw->staging + off;
    if (int rc = launch_swap<true>(p, block_ids, nb, stage, j0, cnt, dev_status, sw->kstream))
      return rc;
    PKV_CUDA_RET(cudaEventRecord(sw->ready, sw->kstream));
    PKV_CUDA_RET(cudaStreamWaitEvent(sw->cstream, sw->ready, 0));
    // the chunk is contiguous in the host layout except where it crosses K -> V
    int64_t j = j0;
    while (j < j0 + cnt) {
      const int64_t end = (j < per_kv) ? std::min(j0 + cnt, per_kv) : j0 + cnt;
      PKV_CUDA_RET(cudaMemcpyAsync(host_seg(hk, hv, j, per_kv, bb), stage + (j - j0) * bb,
                                   size_t((end - j) * bb), cudaMemcpyDeviceToHost, sw->cstream));
      j = end;
    }
    if (int rc = stage_release(sw, off, size_t(cnt * bb), sw->cstream)) return rc;
  }
  // later compute-stream work (writes into the freed blocks) waits for the reads only
  PKV_CUDA_RET(cudaEventRecord(sw->ev_kdone, sw->kstream));
  PKV_CUDA_RET(cudaStreamWaitEvent(cs, sw->ev_kdone, 0));
  return new_ticket(sw, sw->cstream, ticket);
}

extern "C" int pkv_swap_in(pkv_swapper* sw, const pkv_pool* pool, const int32_t* block_ids,
                           int64_t nb, const void* host_k, const void* host_v,
                           void* compute_stream, int32_t* dev_status, uint64_t* ticket) {
  if (int rc = check_swapper(sw)) return rc;
  if (int rc = check_pool(pool)) return rc;
  if (nb < 0) return fail(PKV_ERR_ARG, "nb must be >= 0");
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  if (nb == 0) return new_ticket(sw, sw->kstream, ticket);
  if (!block_ids || !host_k || !host_v) return fail(PKV_ERR_ARG, "block_ids and host buffers must be non-NULL");
  const pkv_pool& p = *pool;
  const int64_t bb = block_bytes(p);
  const int64_t chunk = int64_t(sw->chunk_bytes) / bb;
  if (chunk < 1) return fail(PKV_ERR_ARG, "staging half smaller than one block");
  const int64_t per_kv = int64_t(p.num_layers) * nb, segs = 2 * per_kv;
  char* hk = const_cast<char*>(static_cast<const char*>(host_k));
  char* hv = const_cast<char*>(static_cast<const char*>(host_v));

  // the destination blocks may still be read by queued compute work
  PKV_CUDA_RET(cudaEventRecord(sw->ev_start, cs));
  PKV_CUDA_RET(cudaStreamWaitEvent(sw->kstream, sw->ev_start, 0));
  for (int64_t j0 = 0; j0 < segs; j0 += chunk) {
    const int64_t cnt = std::min(chunk, segs - j0);
    size_t off = 0;
    if (int rc = stage_alloc(sw, size_t(cnt * bb), sw->cstream, &off)) return rc;
    char* stage = sw->staging + off;
    int64_t j = j0;
    while (j < j0 + cnt) {
      const int64_t end = (j < per_kv) ? std::min(j0 + cnt, per_kv) : j0 + cnt;
      PKV_CUDA_RET(cudaMemcpyAsync(stage + (j - j0) * bb, host_seg(hk, hv, j, per_kv, bb),
                                   size_t((end - j) * bb), cudaMemcpyHostToDevice, sw->cstream));
      j = end;
    }
    PKV_CUDA_RET(cudaEventRecord(sw->ready, sw->cstream));
    PKV_CUDA_RET(cudaStreamWaitEvent(sw->kstream, sw->ready, 0));
    if (int rc = launch_swap<false>(p, block_ids, nb, stage, j0, cnt, dev_status, sw->kstream))
      return rc;
    if (int rc = stage_release(sw, off, size_t(cnt * bb), sw->kstream)) return rc;
  }
  PKV_CUDA_RET(cudaEventRecord(sw->ev_kdone, sw->kstream));
  PKV_CUDA_RET(cudaStreamWaitEvent(cs, sw->ev_kdone, 0));
  return new_ticket(sw, sw->kstream, ticket);
}

extern "C" int pkv_swapper_wait(pkv_swapper* sw, uint64_t ticket) {
  if (!sw) return fail(PKV_ERR_ARG, "swapper is NULL");
  if (ticket == 0) {
    PKV_CUDA_RET(cudaStreamSynchronize(sw->kstream));
    PKV_CUDA_RET(cudaStreamSynchronize(sw->cstream));
    for (auto& kv : sw->tickets) cudaEventDestroy(kv.second);
    sw->tickets.clear();
    return PKV_OK;
  }
  auto it = sw->tickets.find(ticket);
  if (it == sw->tickets.end()) return PKV_OK;  // already waited: complete
  PKV_CUDA_RET(cudaEventSynchronize(it->second));
  cudaEventDestroy(it->second);
  sw->tickets.erase(it);
  return PKV_OK;
}

extern "C" int pkv_swapper_done(pkv_swapper* sw, uint64_t ticket) {
  if (!sw) return 0;
  auto it = sw->tickets.find(ticket);
  if (it == sw->tickets.end()) return 1;
  cudaError_t e = cudaEventQuery(it->second);
  if (e == cudaSuccess) {
    cudaEventDestroy(it->second);
    sw->tickets.erase(it);
    return 1;
  }
  if (e != cudaErrorNotReady) cuda_fail(e, "cudaEventQuery");
  return 0;
}
