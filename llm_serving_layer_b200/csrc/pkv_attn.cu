// pkv_attn.cu — paged attention over CSR block tables.
//
// Three kernels:
//   plan_kernel     once per step: expands the CSR page table into one 8-byte
//                   descriptor per page {page id, seq | first | last | valid},
//                   validates it, zeroes the split-K merge counters.
//   decode_kernel   q_len == 1 per sequence, fp16/bf16 pools, head_dim 64,
//                   16-token pages. A persistent grid splits the step's pages
//                   into equal contiguous ranges (one per CTA), so load balance
//                   is exact whatever the length skew; one warp per KV head
//                   streams its [16 x 64] K and V page tiles through a
//                   per-warp TMA ring (128B-swizzled, mbarrier-completed) and
//                   does the math on tensor cores (S^T = K.Q^T, O^T += V^T.P^T,
//                   m16n8k16, fp32 accumulate) with an fp32 online softmax.
//                   A sequence cut by a range boundary leaves a piece at each
//                   end of the ranges it touches; the consumer warps hand their
//                   heads' piece to the CTA's merge warp through shared memory
//                   and move on, and the merge warp publishes it, counts it in
//                   (one atomic counter per sequence) and, if that completes
//                   the count, merges the sequence's pieces — off the
//                   streaming warps' path. A range's cut pieces are processed
//                   first, so their merges overlap the rest of its pages.
//   generic_kernel  any geometry / dtype the tensor-core kernels (decode here,
//                   prefill in pkv_prefill.cu) do not take: one warp per
//                   (token, query head), CUDA cores.
#include <algorithm>
#include <array>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int DK_D = 64;       // head_dim of the decode kernel
constexpr int DK_P = 16;       // tokens per page of the decode kernel
constexpr int DK_NST = 6;                  // default ring depth (pages in flight per CTA)
constexpr int DK_KV_MAX = 8;               // KV heads of the decode kernel (one consumer warp each)
constexpr int DK_WMERGE = 4;               // split-K pieces fetched per round of loads in a merge
constexpr int DK_U = 2;                    // pages folded per online-softmax update
constexpr int DK_PREFETCH = 8;             // pages a CTA prefetches into L2 before the earlier kernel is done
#ifndef DK_PRODUCER_SLEEP_NS
#define DK_PRODUCER_SLEEP_NS 64            // producer back-off while the ring is full
#endif
constexpr int DK_MAXNREG = 168;            // 10 warps: <= 3 per SM sub-partition x 32 x 168 <= 16K registers

// ---------------------------------------------------------------- workspace
struct WsLayout {
  size_t page_desc = 0;  // int4[total_pages]
  size_t counters = 0;   // int32[n_seqs]: split pieces counted in, per sequence
  size_t partial_o = 0;   // float[2 * grid][n_heads][D]
  size_t partial_ml = 0;  // float2[2 * grid][n_heads]
  size_t n_tiles = 0;     // int32[3]: prefill tiles planned, the lean prefill kernel's claim and exit counters (prefill layout only)
  size_t p_dec = 0;       // int64: decode-row pages listed in a mixed batch (prefill layout only)
  size_t rows = 0;        // int32[n_seqs]: their q / out rows (prefill layout only)
  size_t tiles = 0;       // int2[tiles_cap] {seq, first token} (prefill layout only)
  size_t total = 0;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// tiles_cap > 0 appends the prefill tile list after the decode regions (whose
// offsets do not depend on it).
WsLayout ws_layout(int n_heads, int n_seqs, int64_t total_pages, int max_grid, int head_dim,
                   int64_t tiles_cap = 0) {
  WsLayout w;
  size_t off = 0;
  w.page_desc = off;
  off = align256(off + sizeof(int4) * size_t(std::max<int64_t>(total_pages, 1)));
  w.counters = off;
  off = align256(off + sizeof(int32_t) * size_t(std::max(n_seqs, 1)));
  w.partial_o = off;
  off = align256(off + sizeof(float) * size_t(2) * max_grid * n_heads * head_dim);
  w.partial_ml = off;
  off = align256(off + sizeof(float2) * size_t(2) * max_grid * n_heads);
  if (tiles_cap > 0) {
    w.n_tiles = off;
    off = align256(off + 3 * sizeof(int32_t));
    w.p_dec = off;
    off = align256(off + sizeof(int64_t));
    w.rows = off;
    off = align256(off + sizeof(int32_t) * size_t(std::max(n_seqs, 1)));
    w.tiles = off;
    off = align256(off + sizeof(int2) * size_t(tiles_cap));
  }
  w.total = off;
  return w;
}

// ---------------------------------------------------------------- plan
// page_desc[p] = {page id, (seq << 7) | (first << 6) | (last << 5) | valid,
//                 first page of seq, one past its last page}
__global__ void plan_kernel(const int32_t* __restrict__ kv_indptr,
                            const int32_t* __restrict__ kv_indices,
                            const int32_t* __restrict__ last_page_len,
                            const int32_t* __restrict__ kv_lens,
                            const int32_t* __restrict__ cu_q, int n_seqs, int64_t total_pages,
                            int block_size, int64_t num_blocks, int4* __restrict__ desc,
                            int32_t* __restrict__ counters, int check_decode, int32_t* st) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_seqs) return;
  const int s = warp;
  if (lane == 0) counters[s] = 0;
  const int64_t a = kv_indptr[s], b = kv_indptr[s + 1];
  const int lpl = last_page_len[s];
  bool bad = (a > b) || (b > total_pages) || (lpl < 1) || (lpl > block_size);
  if (s == n_seqs - 1 && b != total_pages) bad = true;
  if (kv_lens && !bad) {
    const int64_t kv = kv_lens[s];
    const int64_t pages = b - a;
    if (pages != (kv + block_size - 1) / block_size || (pages - 1) * block_size + lpl != kv) bad = true;
  }
  if (check_decode && cu_q[s + 1] - cu_q[s] != 1) {
    if (lane == 0) flag(st, PKV_DEV_QLEN_BAD);
  }
  if (bad) {
    if (lane == 0) flag(st, PKV_DEV_META_BAD);
  } else {
    for (int64_t p = a + lane; p < b; p += 32) {
      const int id = kv_indices[p];
      if (id < 0 || id >= num_blocks) flag(st, PKV_DEV_SLOT_OOB);
      const int first = (p == a), last = (p == b - 1);
      const int valid = last ? lpl : block_size;
      desc[p] = make_int4(id, (s << 7) | (first << 6) | (last << 5) | valid, int(a), int(b));
    }
  }
  // The decode kernel reads the descriptors before its griddepcontrol.wait (it
  // starts only once this kernel has completed, which never triggers its
  // dependents early): the stores are made visible at GPU scope before the
  // block exits.
  __threadfence();
}

// ---------------------------------------------------------------- decode
struct DecodeArgs {
  const void* q;
  void* out;
  const int4* desc;
  float* partial_o;    // [2 * grid][n_heads][D]   O / l of each split piece
  float2* partial_ml;  // [2 * grid][n_heads]      (m, l) of each split piece
  int32_t* counters;
  int32_t* st;
  const int32_t* rows;   // q / out row of each listed sequence (NULL: row == sequence index)
  const int64_t* p_dev;  // pages listed, read on the device (NULL: total_pages)
  // Fused KV-append (knew NULL: none). Row r's new token (knew/vnew[r], [n_kv][64])
  // is written to its pool slot slots[r] and patched into the staged copy of the
  // sequence's last page, where it must be the last written position.
  const void* knew;
  const void* vnew;
  const int32_t* slots;
  char* k_slab;          // this layer's K / V slab (slot * row_bytes addresses a row)
  char* v_slab;
  int64_t n_slots;
  // Fused rotary embedding (rcos NULL: none; only with the fused KV-append): the
  // q row and the new K row of token `row` are rotated at position positions[row]
  // by the angles whose cosines / sines are rcos / rsin[pos][0 .. 31] (pairs
  // (i, i + 32) of each head), positions outside [0, rmax) flagged.
  const int64_t* positions = nullptr;
  const float* rcos = nullptr;
  const float* rsin = nullptr;
  int64_t rmax = 0;
  int64_t total_pages;   // capacity of desc (and the page count when p_dev is NULL)
  int n_seqs;
  int n_rows;            // rows of q / out
  int n_heads;
  int layer;
  float scale_log2;
  int prefetch;          // pages of the range warmed in L2 before the earlier kernel completed (<= 32)
};

__host__ __device__ constexpr size_t bar_bytes(int n_warps, int nst) {
  return (size_t(n_warps) * nst * 8 + 127) & ~size_t(127);
}

// index of the CTA whose page range [c*P/G, (c+1)*P/G) contains page p
__device__ __forceinline__ int cta_of(int64_t p, int64_t P, int G) {
  return int(((p + 1) * G + P - 1) / P) - 1;
}

template <typename T, int GROUPS>
__device__ __forceinline__ void load_q_frag(const T* __restrict__ q, int row, int n_heads, int h,
                                            int g, int c4, uint32_t (&qb)[4][2]) {
  if (g < GROUPS) {
    const T* qr = q + (int64_t(row) * n_heads + h * GROUPS + g) * DK_D + 2 * c4;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qb[ks][0] = __ldg(reinterpret_cast<const uint32_t*>(qr + ks * 16));
      qb[ks][1] = __ldg(reinterpret_cast<const uint32_t*>(qr + ks * 16 + 8));
    }
  } else {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) qb[ks][0] = qb[ks][1] = 0u;
  }
}

// Rotary embedding of a q fragment (see load_q_frag): the lane holds dims
// 2*c4 + 16*ks + {0, 1} in qb[ks][0] and 2*c4 + 16*ks + 8 + {0, 1} in
// qb[ks][1]; dim i < 32 pairs with dim i + 32, which the same lane holds in
// qb[ks + 2]. cs / sn: the token's 32 cosines / sines.
template <typename T>
__device__ __forceinline__ void rope_q_frag(uint32_t (&qb)[4][2], int c4, const float* cs, const float* sn) {
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int i = 2 * c4 + 16 * ks + 8 * hf;
      const float2 c = __ldg(reinterpret_cast<const float2*>(cs + i));
      const float2 sv = __ldg(reinterpret_cast<const float2*>(sn + i));
      float2 lo = unpack2<T>(qb[ks][hf]), hi = unpack2<T>(qb[ks + 2][hf]);
      rope_pair(lo.x, hi.x, c.x, sv.x);
      rope_pair(lo.y, hi.y, c.y, sv.y);
      qb[ks][hf] = pack2<T>(lo.x, lo.y);
      qb[ks + 2][hf] = pack2<T>(hi.x, hi.y);
    }
}

// Consumer warp h merges the split-K pieces in CTAs cf..cl of a sequence
// (output row `row`) for its query heads h*GROUPS .. h*GROUPS + GROUPS - 1. Its
// own CTA's piece (CTA `own`) is still in the handoff slot: `ostage` (O/l, fp32,
// [GROUPS][64], this warp's heads) and `oml` ((m, l) per head); every other
// piece's O/l and (m, l) are read from the workspace, DK_WMERGE pieces per round
// of loads. Pieces are folded in
// CTA order with weights l * 2^(m - M) whichever warp merges, so the result is
// the same bits run after run. Lane `lane` owns elements [lane*PER, lane*PER + PER).
template <typename T, int GROUPS>
__device__ __forceinline__ void merge_warp(const DecodeArgs& a, int row, int h, int own, int64_t fa,
                                           int cf, int cl, int64_t P, int G, const float* ostage,
                                           const float2* oml, int lane) {
  constexpr int PER = GROUPS * DK_D / 32;  // 2, 4, 8 or 16 elements per lane
  const int nh = a.n_heads;
  const int e0 = lane * PER;
  const int j = e0 / DK_D;
  auto slot_of = [&](int cc) { return 2 * cc + ((cc == cf && fa > int64_t(cc) * P / G) ? 1 : 0); };
  float acc[PER];
#pragma unroll
  for (int r = 0; r < PER; ++r) acc[r] = 0.f;
  float M = -1e30f, W = 0.f;
  for (int k0 = cf; k0 <= cl; k0 += DK_WMERGE) {
    float2 ml[DK_WMERGE];
    float v[DK_WMERGE][PER];
#pragma unroll
    for (int u = 0; u < DK_WMERGE; ++u) {
      const int cc = k0 + u;
      ml[u] = make_float2(-1e30f, 0.f);
#pragma unroll
      for (int r = 0; r < PER; ++r) v[u][r] = 0.f;
      if (cc == own) {
        ml[u] = oml[j];
#pragma unroll
        for (int r = 0; r < PER; ++r) v[u][r] = ostage[e0 + r];
      } else if (cc <= cl) {
        const size_t sl = size_t(slot_of(cc));
        ml[u] = __ldcg(a.partial_ml + sl * nh + h * GROUPS + j);
        const float* po = a.partial_o + (sl * nh + h * GROUPS) * DK_D + e0;
        if constexpr (PER >= 4) {
#pragma unroll
          for (int r = 0; r < PER; r += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(po + r));
            v[u][r] = x.x; v[u][r + 1] = x.y; v[u][r + 2] = x.z; v[u][r + 3] = x.w;
          }
        } else {
          const float2 x = __ldcg(reinterpret_cast<const float2*>(po));
          v[u][0] = x.x; v[u][1] = x.y;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < DK_WMERGE; ++u) {
      if (ml[u].y <= 0.f) continue;  // not a piece of this merge (or an empty one)
      const float Mn = fmaxf(M, ml[u].x);
      const float cs = ex2(M - Mn), cu = ml[u].y * ex2(ml[u].x - Mn);
#pragma unroll
      for (int r = 0; r < PER; ++r) acc[r] = acc[r] * cs + cu * v[u][r];
      W = W * cs + cu;
      M = Mn;
    }
  }
  const float inv = 1.f / W;
  T* dst = static_cast<T*>(a.out) + (int64_t(row) * nh + h * GROUPS) * DK_D + e0;
  uint32_t pk[PER / 2];
#pragma unroll
  for (int r = 0; r < PER; r += 2) pk[r / 2] = MmaOp<T>::pack(acc[r] * inv, acc[r + 1] * inv);
  if constexpr (PER == 16) {
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  } else if constexpr (PER == 8) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  } else if constexpr (PER == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(pk[0], pk[1]);
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pk[0];
  }
}

// Attention of one warp's KV head over U consecutive pages of one sequence,
// folded into the running (m, l, O) state with one online-softmax update.
// kb[u] / vb[u]: shared addresses of page u's [16 tok x 64] K / V tiles (128B
// swizzled); only the last page may be partial (valid_last tokens).
template <typename T, int U>
__device__ __forceinline__ void attend_pages(const uint32_t (&kb)[U], const uint32_t (&vb)[U],
                                             int valid_last, const uint32_t (&qb)[4][2],
                                             float (&o)[4][4], float& m0, float& m1, float& l0,
                                             float& l1, float scale_log2, int k_tok, int k_chk,
                                             int v_tok, int v_chk, int g) {
  // S^T[16 tok x 8 heads] = K[16 x 64] . Q^T[64 x 8], per page
  float s[U][4];
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[u][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t af[4];
      const int chunk = 2 * ks + k_chk;
      ldsm_x4(af[0], af[1], af[2], af[3], kb[u] + k_tok * 128 + ((chunk ^ (k_tok & 7)) << 4));
      MmaOp<T>::run(s[u], af, qb[ks][0], qb[ks][1]);
    }
  }
  // rows g and g+8 are tokens, columns 2*c4 and 2*c4+1 heads of the group
  const bool v0 = g < valid_last, v1 = (g + 8) < valid_last;
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const bool a0 = (u < U - 1) || v0, a1 = (u < U - 1) || v1;
    s[u][0] = a0 ? s[u][0] * scale_log2 : -INFINITY;
    s[u][1] = a0 ? s[u][1] * scale_log2 : -INFINITY;
    s[u][2] = a1 ? s[u][2] * scale_log2 : -INFINITY;
    s[u][3] = a1 ? s[u][3] * scale_log2 : -INFINITY;
    mx0 = fmaxf(mx0, fmaxf(s[u][0], s[u][2]));
    mx1 = fmaxf(mx1, fmaxf(s[u][1], s[u][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
  const float al0 = ex2(m0 - mn0), al1 = ex2(m1 - mn1);
  m0 = mn0;
  m1 = mn1;
  float ls0 = 0.f, ls1 = 0.f;
  uint32_t pb[U][2];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const float p00 = ex2(s[u][0] - mn0), p01 = ex2(s[u][1] - mn1);
    const float p10 = ex2(s[u][2] - mn0), p11 = ex2(s[u][3] - mn1);
    ls0 += p00 + p10;
    ls1 += p01 + p11;
    pb[u][0] = movmatrix_t(MmaOp<T>::pack(p00, p01));
    pb[u][1] = movmatrix_t(MmaOp<T>::pack(p10, p11));
  }
  l0 = l0 * al0 + ls0;
  l1 = l1 * al1 + ls1;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
    o[mt][0] *= al0;
    o[mt][2] *= al0;
    o[mt][1] *= al1;
    o[mt][3] *= al1;
  }
  // O^T[64 dims x 8 heads] += V^T[64 x 16] . P^T[16 x 8], per page
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t af[4];
      const int chunk = 2 * mt + v_chk;
      ldsm_x4_t(af[0], af[1], af[2], af[3], vb[u] + v_tok * 128 + ((chunk ^ (v_tok & 7)) << 4));
      MmaOp<T>::run(o[mt], af, pb[u][0], pb[u][1]);
    }
  }
}

// One CTA = one consumer warp per KV head + one producer warp. The producer
// streams whole pages: one TMA box per page for K and one for V, each the full
// contiguous 16 KiB [16 tok][8 heads][64] page, read through a permuted view of
// the pool (dims D, T, H) so that it lands in shared memory as [head][tok][64]
// with the 128B swizzle keyed on the token (conflict-free ldmatrix over a
// head's 16 tokens). Consumer warp h reads its head's 2 KiB slice of each stage
// and walks the range sequence piece by sequence piece, DK_U pages per
// online-softmax update. A range holds at most two pieces cut by its ends (the
// piece at p0 and the one at p1); they are processed first (the one at p1,
// then the one at p0, then the sequences inside), and each consumer warp writes
// its heads' (O/l, m, l) of such a piece into that piece's handoff slot in
// shared memory and moves on. The merge warp takes each slot when all consumer
// warps arrived, publishes it to the workspace, counts it in with one atomic
// per sequence and, if that completed the count, merges the sequence.
// FUSE: the variant with the KV-append folded in (DecodeArgs::knew set); a
// separate instantiation, so the plain decode kernel carries none of its code.
template <typename T, int GROUPS, int NST, bool FUSE>
__global__ void __maxnreg__(DK_MAXNREG) decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                      const DecodeArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_cons = (blockDim.x >> 5) - 2;  // consumer warps == KV heads; then producer, merge warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  constexpr int PAGE = DK_P * DK_D * 8 * 2;  // 16 KiB: one page of one layer, K or V (8 heads)
  constexpr int STAGE = 2 * PAGE;
  unsigned char* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(NST) * STAGE);
  uint64_t* empty = full + NST;
  uint64_t* hbar = empty + NST;  // [2]: the handoff slots' consumer arrivals
  const int nh = a.n_heads;
  float* ostage_all = reinterpret_cast<float*>(smem + size_t(NST) * STAGE + bar_bytes(2, NST + 1));
  float* hand = ostage_all + size_t(nh) * DK_D;                  // [2][n_heads][64] O/l of the cut pieces
  float2* hml = reinterpret_cast<float2*>(hand + size_t(2) * nh * DK_D);  // [2][n_heads] (m, l)
  int4* mjob = reinterpret_cast<int4*>(hml + 2 * nh);            // [2] {row or -1, cf, cl, fa} of a merge
  int* mstate = reinterpret_cast<int*>(mjob + 2);                // [2] 1 once the merge warp decided

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], n_cons);
    }
    mbar_init(&hbar[0], n_cons);
    mbar_init(&hbar[1], n_cons);
    mstate[0] = mstate[1] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  // Up to pdl_wait() this CTA may run while the kernel before it (an append, the
  // previous layer's attention) still runs. It reads only what the step's plan
  // wrote — the plan kernel lets nothing start before it completed — and warms
  // L2 with its first pages, which is harmless whatever the earlier kernel
  // writes (the loads below go through the same L2).
  // Pages to cover: the decode rows of a mixed batch are listed by the plan on
  // the device, so their count is read there (bounded by the descriptor capacity).
  // The ranges are cut over G = min(grid, P) CTAs, so every range is non-empty
  // (a split sequence's pieces are exactly the CTAs cf..cl); surplus CTAs exit.
  // (L2-level loads, ld.global.cg: nothing here may come from a line this SM
  // cached in L1 before the plan rewrote it)
  const int64_t P = a.p_dev ? max(int64_t(0), min(__ldcg(a.p_dev), a.total_pages)) : a.total_pages;
  const int G = int(min(int64_t(gridDim.x), P));
  const int c = blockIdx.x;
  if (c >= G) return;
  const int64_t p0 = int64_t(c) * P / G, p1 = int64_t(c + 1) * P / G;
  if (p0 >= p1) return;
  const int R = int(p1 - p0);

  // Processing order. The range's last sequence (tail piece T) and first
  // sequence (head piece H) may be cut by the range's ends; T is taken first,
  // then H, then the middle M, so that cut pieces are handed to the merge warp
  // early and their merges overlap the consumers' remaining pages.
  const int4 dfirst = __ldcg(a.desc + p0), dlast = __ldcg(a.desc + p1 - 1);
  const int sf = dfirst.y >> 7, sl = dlast.y >> 7;
  int lenT = 0, lenH = 0;
  int64_t hend = p0, tstart = p1;
  if (sf >= 0 && sl >= 0 && sf != sl && dfirst.w > p0 && dfirst.w <= p1 && dlast.z >= p0 && dlast.z < p1) {
    hend = dfirst.w;
    tstart = dlast.z;
    lenT = int(p1 - tstart);
    lenH = int(hend - p0);
  }
  auto pos = [&](int i) -> int64_t {  // processing step -> page index
    if (i < lenT) return tstart + i;
    if (i < lenT + lenH) return p0 + (i - lenT);
    return (lenT ? hend : p0) + (i - lenT - lenH);
  };
  auto seg_end = [&](int i) -> int64_t {  // one past the last page of step i's segment
    if (i < lenT) return p1;
    if (i < lenT + lenH) return hend;
    return lenT ? tstart : p1;
  };
  const int kv_coord = 2 * a.layer;
  if (warp == n_cons && lane < min(R, a.prefetch)) {
    const int id = __ldcg(&a.desc[pos(lane)].x);
    if (id >= 0) {
      tma_prefetch_l2_4d(&tmap, 0, id * DK_P, 0, kv_coord);
      tma_prefetch_l2_4d(&tmap, 0, id * DK_P, 0, kv_coord + 1);
    }
  }
  // The consumer threads warm L2 with the query rows of the range's first
  // sequences (the tail piece's first, then from the head): a hint, so it may
  // run before the wait (the loads after it read through L2, where a later
  // write by an earlier kernel lands too). One 128-byte row per head.
  if (warp < n_cons && sf >= 0 && sl >= sf) {
    const int tid = warp * 32 + lane, k = tid / a.n_heads, hh = tid % a.n_heads;
    const int sq = k == 0 ? sl : sf + k - 1;
    if (sq <= sl && sq < a.n_seqs) {
      const int row = a.rows ? __ldcg(a.rows + sq) : sq;
      if (row >= 0 && row < a.n_rows)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const T*>(a.q) +
                                                       (int64_t(row) * a.n_heads + hh) * DK_D));
    }
  }
  // The producer also loads the ring's first stages now, up to the first page
  // that is the last page of its sequence: the kernels allowed to run ahead
  // of this one (the append, the RoPE rotation, attention launches) write the
  // pool only at the step's new rows, which lie in the sequences' last pages.
  int pre = 0;
  if (warp == n_cons) {
    if (lane == 0) {
      for (int i = 0; i < min(R, NST); ++i) {
        const int4 d = __ldcg(a.desc + pos(i));
        if ((d.y >> 5) & 1) break;
        unsigned char* dst = stages + size_t(i) * STAGE;
        mbar_arrive_expect_tx(&full[i], 2u * n_cons * DK_P * DK_D * 2);
        tma_load_4d(dst, &tmap, &full[i], 0, d.x * DK_P, 0, kv_coord);
        tma_load_4d(dst + PAGE, &tmap, &full[i], 0, d.x * DK_P, 0, kv_coord + 1);
        pre = i + 1;
      }
    }
    pre = __shfl_sync(0xffffffffu, pre, 0);
  }
  pdl_wait();  // q, this step's appended rows and the split-K counters are written by earlier kernels
  // page descriptors: lane j holds window entries [wb + j] (cur) and [wb + 32 + j] (nxt)
  int wb = 0;
  int4 dcur = make_int4(-1, -1, -1, -1), dnxt = make_int4(-1, -1, -1, -1);
  if (lane < R) dcur = a.desc[pos(lane)];
  if (32 + lane < R) dnxt = a.desc[pos(32 + lane)];
  auto desc_at = [&](int i) -> int4 {  // uniform i in [wb, wb + 64)
    const bool in_cur = i < wb + 32;
    int4 d;
    d.x = __shfl_sync(0xffffffffu, in_cur ? dcur.x : dnxt.x, i & 31);
    d.y = __shfl_sync(0xffffffffu, in_cur ? dcur.y : dnxt.y, i & 31);
    d.z = __shfl_sync(0xffffffffu, in_cur ? dcur.z : dnxt.z, i & 31);
    d.w = __shfl_sync(0xffffffffu, in_cur ? dcur.w : dnxt.w, i & 31);
    return d;
  };
  auto slide_to = [&](int i) {  // make [i, i + 32) resident (i advances by <= 32)
    while (i >= wb + 32) {
      wb += 32;
      dcur = dnxt;
      dnxt = make_int4(-1, -1, -1, -1);
      if (wb + 32 + lane < R) dnxt = a.desc[pos(wb + 32 + lane)];
    }
  };

  auto row_ok = [&](const int4& d, int& row) -> bool {  // the consumers' test of a piece's first page
    const int sq = d.y >> 7;
    row = (sq >= 0 && sq < a.n_seqs) ? (a.rows ? __ldg(a.rows + sq) : sq) : -1;
    return row >= 0 && row < a.n_rows && (d.y & 31) >= 1 && (d.y & 31) <= DK_P;
  };

  // the range's pieces cut by its ends: A (the piece at p0, handoff slot 0) and
  // B (the piece at p1, slot 1)
  int rA, rB;
  const bool cutA = row_ok(dfirst, rA) && (dfirst.z < p0 || dfirst.w > p1);
  const bool cutB = sl != sf && row_ok(dlast, rB) && dlast.w > p1;

  if (warp == n_cons + 1) {
    // ---------------- merge warp: publish each cut piece, count it in, and if
    // that completed the sequence, post the merge for the consumer warps
    for (int t = 0; t < 2; ++t) {
      const int slot = (lenT > 0) ? 1 - t : t;  // in processing order: T (slot 1) first when reordered
      if (!(slot == 0 ? cutA : cutB)) continue;
      const int4 d = slot == 0 ? dfirst : dlast;
      const int seq = d.y >> 7, row = slot == 0 ? rA : rB;
      const int64_t fa = d.z, fb = d.w;
      const int cf = cta_of(fa, P, G), cl = cta_of(fb - 1, P, G);
      int job_row = -1;
      if (mbar_wait_bounded_sleepy(&hbar[slot], 0, a.st, DK_PRODUCER_SLEEP_NS)) {
        const float* ho = hand + size_t(slot) * nh * DK_D;
        const float2* hm = hml + size_t(slot) * nh;
        float* po = a.partial_o + size_t(2 * c + slot) * nh * DK_D;
        for (int e = lane * 4; e < nh * DK_D; e += 32 * 4)
          __stcg(reinterpret_cast<float4*>(po + e), *reinterpret_cast<const float4*>(ho + e));
        for (int j = lane; j < nh; j += 32) __stcg(a.partial_ml + size_t(2 * c + slot) * nh + j, hm[j]);
        __syncwarp();
        int prev = 0;
        int32_t* cnt = a.counters + seq;
        if (lane == 0) asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt) : "memory");
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == cl - cf) {  // every piece is in: this CTA merges; the count restarts at 0
          job_row = row;
          if (lane == 0) *cnt = 0;
        }
      }
      if (lane == 0) {
        mjob[slot] = make_int4(job_row, cf, cl, int(fa));
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&mstate[slot]) = 1;
      }
      __syncwarp();
    }
    return;
  }

  if (warp == n_cons) {
    // ---------------- producer warp
    bool dead = false;
    for (int i = pre; i < R; ++i) {
      slide_to(i);
      const int4 d = desc_at(i);
      const int st = i % NST;
      if constexpr (FUSE) {
        // Fused KV-append: before the TMA of a sequence's last page, the warp
        // writes the sequence's new K/V row (all heads) to its slot and fences
        // the stores for the async proxy, so the page lands with the token in
        // place. The slot must be the page's last written position.
        const int seq = d.y >> 7;
        if (((d.y >> 5) & 1) && seq >= 0 && seq < a.n_seqs) {
          const int row = a.rows ? __ldg(a.rows + seq) : seq;
          if (row >= 0 && row < a.n_rows) {
            const int slot = __ldg(a.slots + row);
            const bool in_pool = slot >= 0 && slot < a.n_slots;
            if (lane == 0 && slot != d.x * DK_P + (d.y & 31) - 1)
              flag(a.st, in_pool ? PKV_DEV_META_BAD : PKV_DEV_SLOT_OOB);
            if (in_pool) {
              const int64_t rb = int64_t(n_cons) * DK_D * sizeof(T);  // one token row, all heads
              const uint4* ks = reinterpret_cast<const uint4*>(static_cast<const char*>(a.knew) + row * rb);
              const uint4* vs = reinterpret_cast<const uint4*>(static_cast<const char*>(a.vnew) + row * rb);
              uint4* kd = reinterpret_cast<uint4*>(a.k_slab + slot * rb);
              uint4* vd = reinterpret_cast<uint4*>(a.v_slab + slot * rb);
              const float* cs = nullptr;
              const float* sn = nullptr;
              if (a.rcos) {
                const int64_t tp = __ldg(a.positions + row);
                if (tp >= 0 && tp < a.rmax) {
                  cs = a.rcos + tp * (DK_D / 2);
                  sn = a.rsin + tp * (DK_D / 2);
                } else if (lane == 0) {
                  flag(a.st, PKV_DEV_META_BAD);  // the row is stored unrotated
                }
              }
              if (cs) {
                // lane = (head, chunk j): dims 8j .. 8j + 7 (uint4 j of the head's
                // row) pair with dims 32 + 8j .. (uint4 j + 4)
                const int hh = lane >> 2, j = lane & 3;
                if (hh < n_cons) {
                  const uint4 lo = __ldg(ks + hh * 8 + j), hi = __ldg(ks + hh * 8 + j + 4);
                  const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + 8 * j));
                  const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + 8 * j + 4));
                  const float4 s0 = __ldg(reinterpret_cast<const float4*>(sn + 8 * j));
                  const float4 s1 = __ldg(reinterpret_cast<const float4*>(sn + 8 * j + 4));
                  const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w}, hw[4] = {hi.x, hi.y, hi.z, hi.w};
                  const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                  const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                  uint32_t ol[4], oh[4];
#pragma unroll
                  for (int w2 = 0; w2 < 4; ++w2) {
                    float2 x = unpack2<T>(lw[w2]), y = unpack2<T>(hw[w2]);
                    rope_pair(x.x, y.x, cc[2 * w2], ss[2 * w2]);
                    rope_pair(x.y, y.y, cc[2 * w2 + 1], ss[2 * w2 + 1]);
                    ol[w2] = pack2<T>(x.x, x.y);
                    oh[w2] = pack2<T>(y.x, y.y);
                  }
                  kd[hh * 8 + j] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
                  kd[hh * 8 + j + 4] = make_uint4(oh[0], oh[1], oh[2], oh[3]);
                }
                for (int e = lane; e < int(rb / 16); e += 32) vd[e] = __ldg(vs + e);
              } else {
                for (int e = lane; e < int(rb / 16); e += 32) {
                  kd[e] = __ldg(ks + e);
                  vd[e] = __ldg(vs + e);
                }
              }
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          }
          __syncwarp();
        }
      }
      if (lane == 0 && !dead) {
        if (i >= NST && !mbar_wait_bounded_sleepy(&empty[st], ((i / NST) - 1) & 1, a.st, DK_PRODUCER_SLEEP_NS))
          dead = true;
        if (!dead) {
          unsigned char* dst = stages + size_t(st) * STAGE;
          mbar_arrive_expect_tx(&full[st], 2u * n_cons * DK_P * DK_D * 2);
          // a rejected page (id -1) reads the zero fill of a negative coordinate
          tma_load_4d(dst, &tmap, &full[st], 0, d.x * DK_P, 0, kv_coord);
          tma_load_4d(dst + PAGE, &tmap, &full[st], 0, d.x * DK_P, 0, kv_coord + 1);
        }
      }
      __syncwarp();
    }
    return;
  }

  // ---------------- consumer warp h
  const int h = warp;
  const T* q = static_cast<const T*>(a.q);
  T* out = static_cast<T*>(a.out);
  float* ostage = ostage_all + size_t(h) * GROUPS * DK_D;
  bool dead = false;
  auto wait_full = [&](int i) {
    if (!dead && !mbar_wait_bounded(&full[i % NST], (i / NST) & 1, a.st)) dead = true;
  };
  auto release = [&](int i) {  // hand stage i % NST back to the producer
    if (lane == 0)
      asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[i % NST])) : "memory");
  };
  auto k_addr = [&](int i) -> uint32_t {
    return smem_u32(stages + size_t(i % NST) * STAGE + h * (DK_P * DK_D * 2));
  };
  auto zero_tail = [&](int i, int valid) {  // never let the unwritten tail of a last page reach P.V
    unsigned char* vt = stages + size_t(i % NST) * STAGE + PAGE + h * (DK_P * DK_D * 2);
    for (int r = valid * 8 + lane; r < DK_P * 8; r += 32)
      reinterpret_cast<uint4*>(vt)[r] = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
  };

  // merges posted by the merge warp, done by every consumer warp for its heads:
  // polled between pieces, and waited for (bounded) once the range is done
  int mdone = (cutA ? 0 : 1) | (cutB ? 0 : 2);
  auto run_merges = [&](bool wait) {
    for (int ms = 0; ms < 2; ++ms) {
      if ((mdone >> ms) & 1) continue;
      int ready = 0;
      if (lane == 0) {
        volatile int* f = &mstate[ms];
        ready = *f;
        if (!ready && wait) {
          const uint64_t t0 = globaltimer_ns();
          while (!(ready = *f) && globaltimer_ns() - t0 < 1000000000ull) __nanosleep(64);
          if (!ready) flag(a.st, PKV_DEV_WAIT_TIMEOUT);
        }
      }
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready && !wait) continue;
      mdone |= 1 << ms;
      if (!ready) continue;
      __threadfence_block();
      const int4 j = mjob[ms];
      if (j.x >= 0)
        merge_warp<T, GROUPS>(a, j.x, h, c, j.w, j.y, j.z, P, G,
                              hand + size_t(ms) * nh * DK_D + size_t(h) * GROUPS * DK_D,
                              hml + size_t(ms) * nh + h * GROUPS, lane);
    }
  };

  uint32_t qb[4][2], qn[4][2];
  int nxt_seq = -1, nxt_row = -1;
  auto row_of = [&](int sq) -> int { return a.rows ? __ldg(a.rows + sq) : sq; };
  auto load_q = [&](int row, uint32_t (&dst)[4][2]) {
    load_q_frag<T, GROUPS>(q, row, a.n_heads, h, g, c4, dst);
    if constexpr (FUSE) {
      if (a.rcos && g < GROUPS) {
        const int64_t tp = __ldg(a.positions + row);
        if (tp >= 0 && tp < a.rmax) rope_q_frag<T>(dst, c4, a.rcos + tp * (DK_D / 2), a.rsin + tp * (DK_D / 2));
        else flag(a.st, PKV_DEV_META_BAD);
      }
    }
  };
  const int first_seq = dfirst.y >> 7;  // its piece (if split) uses partial slot 0
  const int k_tok = (lane & 7) + ((lane >> 3) & 1) * 8, k_chk = lane >> 4;
  const int v_tok = (lane & 7) + (lane >> 4) * 8, v_chk = (lane >> 3) & 1;

  int i = 0;
  while (i < R) {
    slide_to(i);
    const int4 d = desc_at(i);
    const int seq = d.y >> 7;
    const int row = (seq >= 0 && seq < a.n_seqs) ? (seq == nxt_seq ? nxt_row : row_of(seq)) : -1;
    if (row < 0 || row >= a.n_rows || (d.y & 31) < 1 || (d.y & 31) > DK_P) {
      // a page of a sequence the plan rejected: drain and release its stage
      if (lane == 0 && !dead) flag(a.st, PKV_DEV_META_BAD);
      wait_full(i);
      __syncwarp();
      release(i);
      ++i;
      continue;
    }
    // this sequence's piece: processing steps [i, i + n)
    const bool seen_first = (d.y >> 6) & 1;
    const int n = int(min(int64_t(d.w), seg_end(i)) - pos(i));
    const bool ends_here = d.w <= p1;
    if (seq == nxt_seq) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) { qb[ks][0] = qn[ks][0]; qb[ks][1] = qn[ks][1]; }
    } else {
      load_q(row, qb);
    }
    // the sequence processed next: H's after T, then each M in turn
    nxt_seq = (i < lenT) ? sf : seq + 1;
    nxt_row = (nxt_seq >= 0 && nxt_seq < a.n_seqs) ? row_of(nxt_seq) : -1;
    if (nxt_row >= 0 && nxt_row < a.n_rows) load_q(nxt_row, qn);
    else nxt_seq = -1;
    float o[4][4];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
    for (int j = 0; j < n; j += DK_U) {
      const int cnt = min(DK_U, n - j);
      slide_to(i + j);
      const int valid = (j + cnt == n && ends_here) ? (desc_at(i + j + cnt - 1).y & 31) : DK_P;
      if (cnt == DK_U) {
        uint32_t kb[DK_U], vb[DK_U];
#pragma unroll
        for (int u = 0; u < DK_U; ++u) {
          wait_full(i + j + u);
          kb[u] = k_addr(i + j + u);
          vb[u] = kb[u] + PAGE;
        }
        if (valid < DK_P) zero_tail(i + j + DK_U - 1, valid);
        attend_pages<T, DK_U>(kb, vb, valid, qb, o, m0, m1, l0, l1, a.scale_log2, k_tok, k_chk,
                              v_tok, v_chk, g);
      } else {
        for (int u = 0; u < cnt; ++u) {
          wait_full(i + j + u);
          const uint32_t kb[1] = {k_addr(i + j + u)};
          const uint32_t vb[1] = {kb[0] + PAGE};
          const int vu = (u == cnt - 1) ? valid : DK_P;
          if (vu < DK_P) zero_tail(i + j + u, vu);
          attend_pages<T, 1>(kb, vb, vu, qb, o, m0, m1, l0, l1, a.scale_log2, k_tok, k_chk, v_tok,
                             v_chk, g);
        }
      }
      // the next TMA into these stages lands after this warp's own stores to them
      if (valid < DK_P) fence_proxy_async_smem();
      __syncwarp();
      for (int u = 0; u < cnt; ++u) release(i + j + u);
    }
    i += n;

    // finalise the piece: normalise (O/l) into this warp's staging slice (a
    // whole sequence) or into its heads' part of the piece's handoff slot
    const bool whole = seen_first && ends_here;
    const int slot = (seq == first_seq) ? 0 : 1;
    float* fin = whole ? ostage : hand + size_t(slot) * nh * DK_D + size_t(h) * GROUPS * DK_D;
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
    }
    const int j0 = 2 * c4, j1 = 2 * c4 + 1;
    const float i0 = 1.f / lt0, i1 = 1.f / lt1;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      const int d0 = mt * 16 + g, d1 = d0 + 8;
      if (j0 < GROUPS) {
        fin[j0 * DK_D + d0] = o[mt][0] * i0;
        fin[j0 * DK_D + d1] = o[mt][2] * i0;
      }
      if (j1 < GROUPS) {
        fin[j1 * DK_D + d0] = o[mt][1] * i1;
        fin[j1 * DK_D + d1] = o[mt][3] * i1;
      }
    }
    if (!whole) {
      // a piece cut by a range end: hand it to the merge warp and move on
      if (g == 0) {
        float2* hm = hml + size_t(slot) * nh + h * GROUPS;
        if (j0 < GROUPS) hm[j0] = make_float2(m0, lt0);
        if (j1 < GROUPS) hm[j1] = make_float2(m1, lt1);
      }
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&hbar[slot])) : "memory");
      run_merges(false);
      continue;
    }
    __syncwarp();
    // the whole sequence lives in this CTA: store it in the pool dtype
    T* dst = out + (int64_t(row) * a.n_heads + h * GROUPS) * DK_D;
    for (int e = lane * 8; e < GROUPS * DK_D; e += 32 * 8) {
      const float4 x = *reinterpret_cast<const float4*>(ostage + e);
      const float4 y = *reinterpret_cast<const float4*>(ostage + e + 4);
      uint4 v;
      v.x = MmaOp<T>::pack(x.x, x.y);
      v.y = MmaOp<T>::pack(x.z, x.w);
      v.z = MmaOp<T>::pack(y.x, y.y);
      v.w = MmaOp<T>::pack(y.z, y.w);
      *reinterpret_cast<uint4*>(dst + e) = v;
    }
    __syncwarp();
    run_merges(false);
  }
  run_merges(true);
}

// ---------------------------------------------------------------- generic
template <typename T>
struct AccOf { using type = float; };
template <>
struct AccOf<double> { using type = double; };

template <typename T>
__device__ __forceinline__ typename AccOf<T>::type ld_acc(const T* p) {
  if constexpr (std::is_same<T, double>::value) return *p;
  else return to_f<T>(*p);
}
template <typename T>
__device__ __forceinline__ T st_cast(typename AccOf<T>::type x) {
  if constexpr (std::is_same<T, double>::value) return x;
  else return from_f<T>(x);
}
__device__ __forceinline__ float acc_exp(float x) { return expf(x); }
__device__ __forceinline__ double acc_exp(double x) { return exp(x); }

struct GenericArgs {
  const char* k_slab;
  const char* v_slab;
  const void* q;
  void* out;
  const int32_t* cu_q;
  const int32_t* kv_lens;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* last_page_len;
  int32_t* st;
  int64_t num_blocks;
  int64_t total_pages;
  int n_seqs, n_tokens, n_heads, n_kv_heads, head_dim, block_size;
  double scale;
};

constexpr int GEN_MAX_DPL = 8;  // head_dim <= 256

template <typename T>
__global__ void __launch_bounds__(256) generic_kernel(const GenericArgs a) {
  using Acc = typename AccOf<T>::type;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= int64_t(a.n_tokens) * a.n_heads) return;
  const int t = int(warp / a.n_heads), hq = int(warp % a.n_heads);
  const int D = a.head_dim, P = a.block_size;
  T* outp = static_cast<T*>(a.out) + (int64_t(t) * a.n_heads + hq) * D;
  // owning sequence: last s with cu_q[s] <= t
  int lo = 0, hi = a.n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int q_len = a.cu_q[s + 1] - a.cu_q[s];
  const int j = t - a.cu_q[s];
  const int64_t pa = a.kv_indptr[s], pb = a.kv_indptr[s + 1];
  const int lpl = a.last_page_len[s];
  const int64_t pages = pb - pa;
  const int64_t kv_len = (pages - 1) * P + lpl;
  bool bad = pages < 1 || pa < 0 || pb > a.total_pages || lpl < 1 || lpl > P || j < 0 || j >= q_len;
  if (!bad && a.kv_lens && a.kv_lens[s] != kv_len) bad = true;
  const int64_t limit = kv_len - q_len + j;  // last visible key (inclusive)
  if (!bad && limit < 0) bad = true;
  if (bad) {
    if (lane == 0) flag(a.st, PKV_DEV_META_BAD);
    for (int d = lane; d < D; d += 32) outp[d] = st_cast<T>(Acc(0));
    return;
  }
  const int kvh = hq / (a.n_heads / a.n_kv_heads);
  const T* qp = static_cast<const T*>(a.q) + (int64_t(t) * a.n_heads + hq) * D;
  const int64_t row_elems = int64_t(a.n_kv_heads) * D;
  const T* ks = reinterpret_cast<const T*>(a.k_slab);
  const T* vs = reinterpret_cast<const T*>(a.v_slab);
  const Acc scale = Acc(a.scale);

  auto key_ptr = [&](const T* slab, int64_t key, bool& ok) -> const T* {
    const int64_t page = a.kv_indices[pa + key / P];
    ok = page >= 0 && page < a.num_blocks;
    if (!ok) return nullptr;
    return slab + ((page * P + key % P) * row_elems + int64_t(kvh) * D);
  };
  auto score = [&](int64_t key, bool& ok) -> Acc {
    const T* kp = key_ptr(ks, key, ok);
    if (!ok) return Acc(0);
    Acc dot = 0;
    for (int d = 0; d < D; ++d) dot += ld_acc(qp + d) * ld_acc(kp + d);
    return dot * scale;
  };

  // pass 1: running max and normaliser over keys [0, limit]
  Acc m = -INFINITY, l = 0;
  bool any_oob = false;
  for (int64_t k0 = 0; k0 <= limit; k0 += 32) {
    const int64_t key = k0 + lane;
    Acc sc = -INFINITY;
    if (key <= limit) {
      bool ok;
      const Acc v = score(key, ok);
      if (ok) sc = v; else any_oob = true;
    }
    Acc cm = sc;
    for (int off = 16; off; off >>= 1) cm = max(cm, __shfl_xor_sync(0xffffffffu, cm, off));
    const Acc mn = max(m, cm);
    Acc e = (sc == -INFINITY) ? Acc(0) : acc_exp(sc - mn);
    for (int off = 16; off; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
    l = (m == -INFINITY ? Acc(0) : l * acc_exp(m - mn)) + e;
    m = mn;
  }
  if (any_oob) flag(a.st, PKV_DEV_SLOT_OOB);
  // pass 2: O = sum_k p_k v_k / l, dims spread over lanes
  Acc acc[GEN_MAX_DPL];
#pragma unroll
  for (int r = 0; r < GEN_MAX_DPL; ++r) acc[r] = 0;
  for (int64_t k0 = 0; k0 <= limit; k0 += 32) {
    const int64_t key = k0 + lane;
    Acc p = 0;
    if (key <= limit) {
      bool ok;
      const Acc v = score(key, ok);
      if (ok) p = acc_exp(v - m);
    }
    const int nk = int((limit - k0 + 1) < 32 ? (limit - k0 + 1) : 32);
    for (int kk = 0; kk < nk; ++kk) {
      const Acc pk = __shfl_sync(0xffffffffu, p, kk);
      bool ok;
      const T* vp = key_ptr(vs, k0 + kk, ok);
      if (!ok) continue;
#pragma unroll
      for (int r = 0; r < GEN_MAX_DPL; ++r) {
        const int d = lane + 32 * r;
        if (d < D) acc[r] += pk * ld_acc(vp + d);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < GEN_MAX_DPL; ++r) {
    const int d = lane + 32 * r;
    if (d < D) outp[d] = st_cast<T>(acc[r] / l);
  }
}

// ---------------------------------------------------------------- host side
struct TmapEntry {
  int device;
  void* base;
  int64_t num_blocks;
  int num_layers, block_size, n_kv_heads, head_dim, dtype, box_heads;
  CUtensorMap map;
};

// box_heads: KV heads per box (the pool's n_kv_heads for whole pages, 1 for one head's slice)
int get_tmap(const pkv_pool& p, CUtensorMap* out, int box_heads) {
  static std::mutex mu;
  static std::vector<TmapEntry> cache;
  int dev = 0;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : cache) {
    if (e.device == dev && e.base == p.base && e.num_blocks == p.num_blocks &&
        e.num_layers == p.num_layers && e.block_size == p.block_size &&
        e.n_kv_heads == p.n_kv_heads && e.head_dim == p.head_dim && e.dtype == p.dtype &&
        e.box_heads == box_heads) {
      *out = e.map;
      return PKV_OK;
    }
  }
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult qr;
    void* fn = nullptr;
    PKV_CUDA_RET(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr));
    if (qr != cudaDriverEntryPointSuccess || !fn)
      return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const int es = elem_size(p.dtype);
  TmapEntry e{dev, p.base, p.num_blocks, p.num_layers, p.block_size, p.n_kv_heads, p.head_dim, p.dtype,
              box_heads, {}};
  // Permuted view of the pool: dims (D, token slot, KV head, layer*2+kv) with
  // strides (elem, row, head_dim*elem, slab). One box = one page of one layer's
  // K or V for box_heads heads, landing in shared memory as [head][token][D].
  const cuuint64_t dims[4] = {cuuint64_t(p.head_dim), cuuint64_t(p.num_blocks) * p.block_size,
                              cuuint64_t(p.n_kv_heads), cuuint64_t(2) * p.num_layers};
  const cuuint64_t strides[3] = {cuuint64_t(row_bytes(p)), cuuint64_t(p.head_dim) * es,
                                 cuuint64_t(slab_bytes(p))};
  const cuuint32_t box[4] = {cuuint32_t(p.head_dim), cuuint32_t(p.block_size), cuuint32_t(box_heads), 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt =
      p.dtype == PKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode(&e.map, dt, 4, p.base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  if (cache.size() > 64) cache.erase(cache.begin());
  cache.push_back(e);
  *out = e.map;
  return PKV_OK;
}

bool decode_supported(const pkv_pool& p, int n_heads) {
  if (p.dtype != PKV_F16 && p.dtype != PKV_BF16) return false;
  if (p.head_dim != DK_D || p.block_size != DK_P) return false;
  if (p.n_kv_heads < 1 || p.n_kv_heads > 8) return false;
  if (n_heads % p.n_kv_heads) return false;
  const int gq = n_heads / p.n_kv_heads;
  return gq == 1 || gq == 2 || gq == 4 || gq == 8;
}

size_t decode_smem(int n_kv_heads, int groups, int nst) {
  const size_t stage = size_t(2) * DK_P * DK_D * 8 * 2;  // K + V page, 8 heads (boxes always 8 wide)
  const size_t nh = size_t(n_kv_heads) * groups;
  // ring, barriers, staging slices, two handoff slots (O/l and (m, l)), merge jobs
  return 1024 + nst * stage + bar_bytes(2, nst + 1) + nh * DK_D * 4 + 2 * nh * DK_D * 4 + 2 * nh * 8 +
         2 * sizeof(int4) + 16;
}

// Ring depth, L2 prefetch depth and CTAs per SM of the decode kernel. Defaults
// are the tuned values; PKV_DECODE_NST (3, 4, 5 or 6), PKV_DECODE_PREFETCH
// (0-32 pages) and PKV_DECODE_CTAS_PER_SM override them for sweeps.
int decode_nst() {
  static int v = [] {
    const char* e = getenv("PKV_DECODE_NST");
    const int n = e ? atoi(e) : DK_NST;
    return (n == 3 || n == 4 || n == 5 || n == 6) ? n : DK_NST;
  }();
  return v;
}
// the deepest ring (<= the requested depth) whose shared memory fits a CTA
int decode_nst_for(int n_kv_heads, int groups) {
  int n = decode_nst();
  while (n > 3 && decode_smem(n_kv_heads, groups, n) > size_t(232448)) --n;
  return n;
}
int decode_prefetch() {
  static int v = [] {
    const char* e = getenv("PKV_DECODE_PREFETCH");
    const int n = e ? atoi(e) : DK_PREFETCH;
    return (n >= 0 && n <= 32) ? n : DK_PREFETCH;
  }();
  return v;
}
int decode_ctas_per_sm_cap() {
  static int v = [] {
    const char* e = getenv("PKV_DECODE_CTAS_PER_SM");
    const int n = e ? atoi(e) : 0;
    return n > 0 ? n : 64;
  }();
  return v;
}

// CTAs of the decode kernel resident per SM, cached per (device, n_kv_heads);
// also raises the kernel's dynamic shared-memory limit on first use per device.
template <typename T, int GROUPS, int NST, bool FUSE>
int decode_grid_limit(int n_kv_heads) {
  static std::mutex mu;
  static std::vector<std::array<int, 9>> occ;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)occ.size() <= dev) occ.resize(dev + 1, std::array<int, 9>{});
  int& o = occ[dev][n_kv_heads];
  if (!o) {
    auto fn = decode_kernel<T, GROUPS, NST, FUSE>;
    const size_t sm = decode_smem(n_kv_heads, GROUPS, NST);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    int v = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, fn, 32 * (n_kv_heads + 2), sm);
    if (e != cudaSuccess) {
      cuda_fail(e, "decode kernel occupancy query");
      return -1;
    }
    o = std::max(1, std::min(v, decode_ctas_per_sm_cap()));
  }
  return o * num_sms();
}

int max_decode_grid() { return num_sms() * 8; }

template <typename T, int GROUPS, int NST, bool FUSE>
int launch_decode_f(const pkv_pool& p, const CUtensorMap& tm, DecodeArgs& a, int64_t total_pages,
                    cudaStream_t s) {
  int limit = decode_grid_limit<T, GROUPS, NST, FUSE>(p.n_kv_heads);
  if (limit <= 0) return PKV_ERR_CUDA;  // message already set
  limit = std::min(limit, max_decode_grid());
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(limit, total_pages)));
  a.prefetch = decode_prefetch();
  PKV_CUDA_RET(launch_kernel(decode_kernel<T, GROUPS, NST, FUSE>, dim3(grid), dim3(32 * (p.n_kv_heads + 2)),
                             decode_smem(p.n_kv_heads, GROUPS, NST), s, true, tm, a));
  return PKV_OK;
}

template <typename T, int GROUPS, int NST, int UNUSED>
int launch_decode_t(const pkv_pool& p, const CUtensorMap& tm, DecodeArgs& a, int64_t tp, cudaStream_t s) {
  return a.knew ? launch_decode_f<T, GROUPS, NST, true>(p, tm, a, tp, s)
                : launch_decode_f<T, GROUPS, NST, false>(p, tm, a, tp, s);
}

template <typename T, int GROUPS>
int launch_decode_n(const pkv_pool& p, const CUtensorMap& tm, DecodeArgs& a, int64_t tp,
                    cudaStream_t s) {
  switch (decode_nst_for(p.n_kv_heads, GROUPS)) {
    case 3: return launch_decode_t<T, GROUPS, 3, 1>(p, tm, a, tp, s);
    case 5: return launch_decode_t<T, GROUPS, 5, 1>(p, tm, a, tp, s);
    case 6: return launch_decode_t<T, GROUPS, 6, 1>(p, tm, a, tp, s);
    default: return launch_decode_t<T, GROUPS, 4, 1>(p, tm, a, tp, s);
  }
}

template <typename T>
int launch_decode_g(const pkv_pool& p, int groups, const CUtensorMap& tm, DecodeArgs& a,
                    int64_t tp, cudaStream_t s) {
  switch (groups) {
    case 1: return launch_decode_n<T, 1>(p, tm, a, tp, s);
    case 2: return launch_decode_n<T, 2>(p, tm, a, tp, s);
    case 4: return launch_decode_n<T, 4>(p, tm, a, tp, s);
    case 8: return launch_decode_n<T, 8>(p, tm, a, tp, s);
  }
  return fail(PKV_ERR_UNSUPPORTED, "decode kernel: unsupported GQA group size");
}

int check_batch(const pkv_pool& p, int32_t n_heads, const pkv_batch* b) {
  if (!b) return fail(PKV_ERR_ARG, "batch descriptor is NULL");
  if (n_heads <= 0 || n_heads % p.n_kv_heads)
    return fail(PKV_ERR_ARG, "n_heads must be a positive multiple of n_kv_heads");
  if (b->n_seqs <= 0) return fail(PKV_ERR_ARG, "batch has no sequences");
  if (b->n_tokens < 0 || b->total_pages < 0) return fail(PKV_ERR_ARG, "negative batch sizes");
  if (!b->cu_query_lens || !b->kv_indptr || !b->kv_last_page_len || (b->total_pages && !b->kv_indices))
    return fail(PKV_ERR_ARG, "batch CSR pointers must be non-NULL");
  if (b->total_pages >= (int64_t(1) << 31)) return fail(PKV_ERR_ARG, "too many pages");
  return PKV_OK;
}

// Workspace layout of a step: the decode regions, plus the prefill tile list
// when the step is not a decode step and the prefill kernel takes it.
WsLayout step_layout(const pkv_pool* pool, int n_heads, int n_seqs, int64_t total_pages, bool decode) {
  const int d = pool ? pool->head_dim : DK_D;
  const int64_t cap = (!decode && pool && prefill_supported(*pool, n_heads))
                          ? prefill_tiles_cap(n_seqs, total_pages) : 0;
  return ws_layout(n_heads, n_seqs, total_pages, max_decode_grid(), d, cap);
}

}  // namespace

int pool_tmap(const pkv_pool& p, CUtensorMap* out) { return get_tmap(p, out, p.n_kv_heads); }
int pool_tmap_head(const pkv_pool& p, CUtensorMap* out) { return get_tmap(p, out, 1); }

}  // namespace pkv

using namespace pkv;

extern "C" size_t pkv_attend_workspace_size(const pkv_pool* pool, int32_t n_heads, int32_t n_seqs,
                                            int64_t total_pages, int32_t decode_hint) {
  return step_layout(pool, n_heads, n_seqs, total_pages, decode_hint == 1).total;
}

extern "C" int pkv_plan(const pkv_pool* pool, int32_t n_heads, const pkv_batch* batch,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  if (int rc = check_batch(*pool, n_heads, batch)) return rc;
  const bool decode = batch->n_tokens == batch->n_seqs;
  if (!decode && !prefill_supported(*pool, n_heads)) return PKV_OK;  // the generic kernel needs no plan
  const WsLayout w = step_layout(pool, n_heads, batch->n_seqs, batch->total_pages, decode);
  if (!workspace || workspace_bytes < w.total)
    return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
  char* ws = static_cast<char*>(workspace);
  if (!decode) {
    // a mixed batch's q_len == 1 rows go to the decode kernel when it takes the geometry
    PrefillMixedPlan mp{reinterpret_cast<int4*>(ws + w.page_desc), reinterpret_cast<int32_t*>(ws + w.counters),
                        reinterpret_cast<int32_t*>(ws + w.rows), reinterpret_cast<int64_t*>(ws + w.p_dec)};
    return prefill_plan(*pool, n_heads, *batch, reinterpret_cast<int2*>(ws + w.tiles),
                        reinterpret_cast<int32_t*>(ws + w.n_tiles), prefill_tiles_cap(batch->n_seqs, batch->total_pages),
                        decode_supported(*pool, n_heads) ? &mp : nullptr, static_cast<cudaStream_t>(stream));
  }
  // every descriptor starts as "no sequence" (-1): pages of a sequence the
  // plan rejects are skipped by the decode kernel instead of read as garbage
  PKV_CUDA_RET(cudaMemsetAsync(ws + w.page_desc, 0xff, sizeof(int4) * size_t(batch->total_pages),
                               static_cast<cudaStream_t>(stream)));
  const int threads = 256;
  const int64_t n_threads = int64_t(batch->n_seqs) * 32;
  plan_kernel<<<unsigned((n_threads + threads - 1) / threads), threads, 0,
                static_cast<cudaStream_t>(stream)>>>(
      batch->kv_indptr, batch->kv_indices, batch->kv_last_page_len, batch->kv_lens,
      batch->cu_query_lens, batch->n_seqs, batch->total_pages, pool->block_size, pool->num_blocks,
      reinterpret_cast<int4*>(ws + w.page_desc), reinterpret_cast<int32_t*>(ws + w.counters),
      1, batch->dev_status);
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

extern "C" int pkv_attend_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads,
                                  const void* q, void* out, float scale, const pkv_batch* batch,
                                  int32_t decode_hint, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (layer < 0 || layer >= p.num_layers)
    return fail(PKV_ERR_ARG, "layer_idx " + std::to_string(layer) + " out of range [0, " +
                                 std::to_string(p.num_layers) + ")");
  if (int rc = check_batch(p, n_heads, batch)) return rc;
  if (!q || !out) return fail(PKV_ERR_ARG, "q and out must be non-NULL");
  if (batch->n_tokens == 0) return PKV_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  if (decode_hint == 1 && decode_supported(p, n_heads)) {
    if (batch->n_tokens != batch->n_seqs)
      return fail(PKV_ERR_ARG, "decode: n_tokens must equal n_seqs (one query per sequence)");
    if (batch->total_pages == 0) return fail(PKV_ERR_ARG, "decode: empty page table");
    const WsLayout w = step_layout(pool, n_heads, batch->n_seqs, batch->total_pages, true);
    if (!workspace || workspace_bytes < w.total)
      return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
      return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
    CUtensorMap tm;
    if (int rc = get_tmap(p, &tm, p.n_kv_heads)) return rc;
    char* ws = static_cast<char*>(workspace);
    DecodeArgs a;
    a.q = q;
    a.out = out;
    a.desc = reinterpret_cast<const int4*>(ws + w.page_desc);
    a.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
    a.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
    a.counters = reinterpret_cast<int32_t*>(ws + w.counters);
    a.st = batch->dev_status;
    a.rows = nullptr;
    a.p_dev = nullptr;
    a.knew = a.vnew = nullptr;
    a.slots = nullptr;
    a.k_slab = a.v_slab = nullptr;
    a.n_slots = 0;
    a.total_pages = batch->total_pages;
    a.n_seqs = batch->n_seqs;
    a.n_rows = batch->n_tokens;
    a.n_heads = n_heads;
    a.layer = layer;
    a.scale_log2 = scale * 1.4426950408889634f;
    const int groups = n_heads / p.n_kv_heads;
    if (p.dtype == PKV_F16) return launch_decode_g<__half>(p, groups, tm, a, batch->total_pages, s);
    return launch_decode_g<__nv_bfloat16>(p, groups, tm, a, batch->total_pages, s);
  }

  if (decode_hint != 1 && batch->n_tokens != batch->n_seqs && prefill_supported(p, n_heads)) {
    const WsLayout w = step_layout(pool, n_heads, batch->n_seqs, batch->total_pages, false);
    if (!workspace || workspace_bytes < w.total)
      return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
    char* ws = static_cast<char*>(workspace);
    if (decode_hint != 2 && decode_supported(p, n_heads) && batch->total_pages > 0) {
      // the q_len == 1 rows the plan listed, on the decode kernel
      if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
      CUtensorMap tm;
      if (int rc = get_tmap(p, &tm, p.n_kv_heads)) return rc;
      DecodeArgs a;
      a.q = q;
      a.out = out;
        a.desc = reinterpret_cast<const int4*>(ws + w.page_desc);
      a.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
      a.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
      a.counters = reinterpret_cast<int32_t*>(ws + w.counters);
      a.st = batch->dev_status;
      a.rows = reinterpret_cast<const int32_t*>(ws + w.rows);
      a.p_dev = reinterpret_cast<const int64_t*>(ws + w.p_dec);
      a.knew = a.vnew = nullptr;
      a.slots = nullptr;
      a.k_slab = a.v_slab = nullptr;
      a.n_slots = 0;
      a.total_pages = batch->total_pages;
      a.n_seqs = batch->n_seqs;
      a.n_rows = batch->n_tokens;
      a.n_heads = n_heads;
      a.layer = layer;
      a.scale_log2 = scale * 1.4426950408889634f;
      const int groups = n_heads / p.n_kv_heads;
      const int rc = p.dtype == PKV_F16 ? launch_decode_g<__half>(p, groups, tm, a, batch->total_pages, s)
                                        : launch_decode_g<__nv_bfloat16>(p, groups, tm, a, batch->total_pages, s);
      if (rc) return rc;
    }
    return prefill_attend(p, layer, n_heads, q, out, scale, *batch, reinterpret_cast<const int2*>(ws + w.tiles),
                          reinterpret_cast<const int32_t*>(ws + w.n_tiles),
                          prefill_tiles_cap(batch->n_seqs, batch->total_pages), s);
  }

  if (p.head_dim > 32 * GEN_MAX_DPL)
    return fail(PKV_ERR_UNSUPPORTED, "head_dim > 256 is not supported");
  GenericArgs g;
  const int64_t sb = slab_bytes(p);
  g.k_slab = static_cast<const char*>(p.base) + (2 * int64_t(layer)) * sb;
  g.v_slab = g.k_slab + sb;
  g.q = q;
  g.out = out;
  g.cu_q = batch->cu_query_lens;
  g.kv_lens = batch->kv_lens;
  g.kv_indptr = batch->kv_indptr;
  g.kv_indices = batch->kv_indices;
  g.last_page_len = batch->kv_last_page_len;
  g.st = batch->dev_status;
  g.num_blocks = p.num_blocks;
  g.total_pages = batch->total_pages;
  g.n_seqs = batch->n_seqs;
  g.n_tokens = batch->n_tokens;
  g.n_heads = n_heads;
  g.n_kv_heads = p.n_kv_heads;
  g.head_dim = p.head_dim;
  g.block_size = p.block_size;
  g.scale = scale;
  const int64_t warps = int64_t(batch->n_tokens) * n_heads;
  const unsigned grid = unsigned((warps * 32 + 255) / 256);
  switch (p.dtype) {
    case PKV_F16: generic_kernel<__half><<<grid, 256, 0, s>>>(g); break;
    case PKV_BF16: generic_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(g); break;
    case PKV_F32: generic_kernel<float><<<grid, 256, 0, s>>>(g); break;
    case PKV_F64: generic_kernel<double><<<grid, 256, 0, s>>>(g); break;
  }
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

extern "C" int pkv_attend_kernel(const pkv_pool* pool, int32_t n_heads, int32_t n_seqs, int32_t n_tokens,
                                 int32_t decode_hint) {
  if (int rc = check_pool(pool)) return -rc;
  if (n_heads <= 0 || n_heads % pool->n_kv_heads) return -fail(PKV_ERR_ARG, "n_heads must be a positive multiple of n_kv_heads");
  if (decode_hint == 1 && decode_supported(*pool, n_heads)) return PKV_KERNEL_DECODE;
  if (decode_hint != 1 && n_tokens != n_seqs && prefill_supported(*pool, n_heads)) return PKV_KERNEL_PREFILL;
  return PKV_KERNEL_GENERIC;
}

namespace {
struct RopeIn {  // fused rotary embedding: none when cos is NULL
  const int64_t* positions;
  const float* cos;
  const float* sin;
  int64_t max_pos;
};

int append_attend_impl(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* k, const void* v,
                       const int32_t* slot_mapping, const void* q, void* out, float scale, const pkv_batch* batch,
                       int32_t decode_hint, void* workspace, size_t workspace_bytes, const RopeIn& rope,
                       void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (layer < 0 || layer >= p.num_layers)
    return fail(PKV_ERR_ARG, "layer_idx " + std::to_string(layer) + " out of range [0, " +
                                 std::to_string(p.num_layers) + ")");
  if (int rc = check_batch(p, n_heads, batch)) return rc;
  if (!k || !v || !slot_mapping) return fail(PKV_ERR_ARG, "k, v and slot_mapping must be non-NULL");
  if (!q || !out) return fail(PKV_ERR_ARG, "q and out must be non-NULL");
  if (batch->n_tokens == 0) return PKV_OK;
  const bool fused = decode_hint == 1 && decode_supported(p, n_heads) && batch->n_tokens == batch->n_seqs &&
                     batch->total_pages > 0 &&
                     ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0;
  if (!fused && rope.cos)
    return fail(PKV_ERR_UNSUPPORTED,
                "the rotary embedding is fused only into a decode batch's single launch (decode_hint 1, the decode "
                "kernel's geometry, 16-byte aligned k and v); rotate q and k with pkv_rope and call "
                "pkv_append_attend_planned");
  if (!fused) {  // the two calls the fused launch replaces
    if (int rc = pkv_append_kv(pool, layer, k, v, slot_mapping, batch->n_tokens, batch->dev_status, stream))
      return rc;
    return pkv_attend_planned(pool, layer, n_heads, q, out, scale, batch, decode_hint, workspace,
                              workspace_bytes, stream);
  }
  const WsLayout w = step_layout(pool, n_heads, batch->n_seqs, batch->total_pages, true);
  if (!workspace || workspace_bytes < w.total)
    return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
  CUtensorMap tm;
  if (int rc = get_tmap(p, &tm, p.n_kv_heads)) return rc;
  char* ws = static_cast<char*>(workspace);
  const int64_t sb = slab_bytes(p);
  DecodeArgs a;
  a.q = q;
  a.out = out;
  a.desc = reinterpret_cast<const int4*>(ws + w.page_desc);
  a.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
  a.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
  a.counters = reinterpret_cast<int32_t*>(ws + w.counters);
  a.st = batch->dev_status;
  a.rows = nullptr;
  a.p_dev = nullptr;
  a.knew = k;
  a.vnew = v;
  a.slots = slot_mapping;
  a.k_slab = static_cast<char*>(p.base) + (2 * int64_t(layer)) * sb;
  a.v_slab = a.k_slab + sb;
  a.n_slots = p.num_blocks * p.block_size;
  a.positions = rope.positions;
  a.rcos = rope.cos;
  a.rsin = rope.sin;
  a.rmax = rope.max_pos;
  a.total_pages = batch->total_pages;
  a.n_seqs = batch->n_seqs;
  a.n_rows = batch->n_tokens;
  a.n_heads = n_heads;
  a.layer = layer;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int groups = n_heads / p.n_kv_heads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.dtype == PKV_F16) return launch_decode_g<__half>(p, groups, tm, a, batch->total_pages, s);
  return launch_decode_g<__nv_bfloat16>(p, groups, tm, a, batch->total_pages, s);
}
}  // namespace

extern "C" int pkv_append_attend_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* k,
                                         const void* v, const int32_t* slot_mapping, const void* q, void* out,
                                         float scale, const pkv_batch* batch, int32_t decode_hint, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  return append_attend_impl(pool, layer, n_heads, k, v, slot_mapping, q, out, scale, batch, decode_hint, workspace,
                            workspace_bytes, RopeIn{nullptr, nullptr, nullptr, 0}, stream);
}

extern "C" int pkv_append_attend_rope_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* k,
                                              const void* v, const int32_t* slot_mapping, const void* q, void* out,
                                              float scale, const pkv_batch* batch, int32_t decode_hint,
                                              void* workspace, size_t workspace_bytes, const int64_t* positions,
                                              const float* rope_cos, const float* rope_sin, int64_t rope_max_pos,
                                              void* stream) {
  if (!positions || !rope_cos || !rope_sin)
    return fail(PKV_ERR_ARG, "positions, rope_cos and rope_sin must be non-NULL");
  if (rope_max_pos <= 0) return fail(PKV_ERR_ARG, "rope_max_pos must be positive");
  if ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15)
    return fail(PKV_ERR_ARG, "rope_cos and rope_sin must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(positions) & 7) return fail(PKV_ERR_ARG, "positions must be 8-byte aligned");
  return append_attend_impl(pool, layer, n_heads, k, v, slot_mapping, q, out, scale, batch, decode_hint, workspace,
                            workspace_bytes, RopeIn{positions, rope_cos, rope_sin, rope_max_pos}, stream);
}

extern "C" int pkv_attend(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* q,
                          void* out, float scale, const pkv_batch* batch, int32_t decode_hint,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (pool && batch && ((decode_hint == 1 && decode_supported(*pool, n_heads)) ||
                        (decode_hint != 1 && batch->n_tokens != batch->n_seqs && prefill_supported(*pool, n_heads)))) {
    if (int rc = pkv_plan(pool, n_heads, batch, workspace, workspace_bytes, stream)) return rc;
  }
  return pkv_attend_planned(pool, layer, n_heads, q, out, scale, batch, decode_hint, workspace,
                            workspace_bytes, stream);
}

// ---------------------------------------------------------------- no-allocation decode
//
// pkv_attend_decode_noalloc: the decode path (plan + split-K decode kernel) for
// callers that cannot allocate device memory — a serving process that hands
// (nearly) all of HBM to its own KV pool and allocates nothing afterwards, or a
// host that owns every device allocation and does not let a plug-in library
// call cudaMalloc. The per-step scratch (page descriptors, split-K counters and
// partials) lives in one file-scope __device__ array instead of a caller's
// workspace.

namespace pkv {
namespace {

// Bytes of the shared scratch: split-K partials for 148 CTAs plus one 16-byte
// descriptor per page leave room for ~340k pages at 32 query heads (~190k at
// 64). Every GPU that loads the library holds this array until the process exits.
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(8) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch for the current device. The host-side
// symbol is only a stand-in, never a device address: the address is looked up
// once per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static std::vector<void*> addr;
  int dev = 0;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)addr.size() <= dev) addr.resize(dev + 1, nullptr);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return PKV_OK;
}

// Upper bound of the decode kernel's grid for this pool (the same occupancy
// query the launch uses), so the scratch layout covers every CTA's partials.
template <typename T, int GROUPS>
int decode_grid_cap_n(const pkv_pool& p) {
  switch (decode_nst_for(p.n_kv_heads, GROUPS)) {
    case 3: return decode_grid_limit<T, GROUPS, 3, false>(p.n_kv_heads);
    case 5: return decode_grid_limit<T, GROUPS, 5, false>(p.n_kv_heads);
    case 6: return decode_grid_limit<T, GROUPS, 6, false>(p.n_kv_heads);
    default: return decode_grid_limit<T, GROUPS, 4, false>(p.n_kv_heads);
  }
}
template <typename T>
int decode_grid_cap(const pkv_pool& p, int groups) {
  switch (groups) {
    case 1: return decode_grid_cap_n<T, 1>(p);
    case 2: return decode_grid_cap_n<T, 2>(p);
    case 4: return decode_grid_cap_n<T, 4>(p);
    default: return decode_grid_cap_n<T, 8>(p);
  }
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_attend_decode_noalloc(const pkv_pool* pool, int32_t layer, int32_t n_heads,
                                         const void* q, void* out, float scale,
                                         const pkv_batch* batch, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  const pkv_pool& p = *pool;
  if (layer < 0 || layer >= p.num_layers)
    return fail(PKV_ERR_ARG, "layer_idx " + std::to_string(layer) + " out of range [0, " +
                                 std::to_string(p.num_layers) + ")");
  if (int rc = check_batch(p, n_heads, batch)) return rc;
  if (!q || !out) return fail(PKV_ERR_ARG, "q and out must be non-NULL");
  if (!decode_supported(p, n_heads))
    return fail(PKV_ERR_UNSUPPORTED, "no-allocation decode needs an fp16/bf16 pool, head_dim 64, "
                                     "16-token pages, <= 8 KV heads and 1/2/4/8 query heads per KV head");
  if (batch->n_tokens != batch->n_seqs)
    return fail(PKV_ERR_ARG, "decode: n_tokens must equal n_seqs (one query per sequence)");
  if (batch->total_pages == 0) return fail(PKV_ERR_ARG, "decode: empty page table");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
  const int groups = n_heads / p.n_kv_heads;
  const int cap = p.dtype == PKV_F16 ? decode_grid_cap<__half>(p, groups)
                                     : decode_grid_cap<__nv_bfloat16>(p, groups);
  if (cap <= 0) return PKV_ERR_CUDA;  // message already set
  const WsLayout w = ws_layout(n_heads, batch->n_seqs, batch->total_pages,
                               std::min(cap, max_decode_grid()), p.head_dim);
  if (w.total > NOALLOC_SCRATCH_BYTES)
    return fail(PKV_ERR_ARG, "batch needs " + std::to_string(w.total) + " bytes of scratch; the "
                             "no-allocation decode has " + std::to_string(NOALLOC_SCRATCH_BYTES) +
                             " (fewer pages or sequences per call, or use pkv_attend with a workspace)");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  char* ws = static_cast<char*>(scratch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // plan: descriptors start at -1, counters are zeroed by the plan kernel, so
  // nothing left in the shared scratch by an earlier call is read
  PKV_CUDA_RET(cudaMemsetAsync(ws + w.page_desc, 0xff, sizeof(int4) * size_t(batch->total_pages), s));
  const int64_t n_threads = int64_t(batch->n_seqs) * 32;
  plan_kernel<<<unsigned((n_threads + 255) / 256), 256, 0, s>>>(
      batch->kv_indptr, batch->kv_indices, batch->kv_last_page_len, batch->kv_lens,
      batch->cu_query_lens, batch->n_seqs, batch->total_pages, p.block_size, p.num_blocks,
      reinterpret_cast<int4*>(ws + w.page_desc), reinterpret_cast<int32_t*>(ws + w.counters), 1,
      batch->dev_status);
  PKV_CUDA_RET(cudaGetLastError());
  CUtensorMap tm;
  if (int rc = get_tmap(p, &tm, p.n_kv_heads)) return rc;
  DecodeArgs a;
  a.q = q;
  a.out = out;
  a.desc = reinterpret_cast<const int4*>(ws + w.page_desc);
  a.partial_o = reinterpret_cast<float*>(ws + w.partial_o);
  a.partial_ml = reinterpret_cast<float2*>(ws + w.partial_ml);
  a.counters = reinterpret_cast<int32_t*>(ws + w.counters);
  a.st = batch->dev_status;
  a.rows = nullptr;
  a.p_dev = nullptr;
  a.knew = a.vnew = nullptr;
  a.slots = nullptr;
  a.k_slab = a.v_slab = nullptr;
  a.n_slots = 0;
  a.total_pages = batch->total_pages;
  a.n_seqs = batch->n_seqs;
  a.n_rows = batch->n_tokens;
  a.n_heads = n_heads;
  a.layer = layer;
  a.scale_log2 = scale * 1.4426950408889634f;
  if (p.dtype == PKV_F16) return launch_decode_g<__half>(p, groups, tm, a, batch->total_pages, s);
  return launch_decode_g<__nv_bfloat16>(p, groups, tm, a, batch->total_pages, s);
}
