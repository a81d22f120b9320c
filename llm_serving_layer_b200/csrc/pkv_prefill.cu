// pkv_prefill.cu — chunked-prefill / mixed-batch attention on tensor cores.
//
// Two kernels:
//   prefill_plan_kernel  once per step (one CTA): cuts every sequence's query
//                        rows into tiles of QT tokens, orders the tiles by the
//                        number of pages they read (longest first) and writes
//                        the tile list into the workspace.
//   prefill_kernel       one CTA per tile, all KV heads: a page ring fed by TMA
//                        (the pool's whole-page [8 heads][16 tok][64] boxes,
//                        128B-swizzled), two consumer warps per KV head, each
//                        with 32 query rows (TPW tokens x the head's GQA group);
//                        S = Q.K^T and O += P.V on m16n8k16 tensor-core MMAs
//                        (fp32 accumulate) with an fp32 online softmax and the
//                        bottom-right causal mask key <= kv_len - q_len + j.
//
// Semantics follow PagedTorchBackend.attend (serving/backends/paged_torch.py:
// 400-485): GQA head h reads KV head h // groups, pages in listed order, the
// mask triu(diag = kv_len - q_len + 1) (paged_torch.py:470-476), and the
// unwritten tail of a sequence's last page never reaches the output.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int PF_D = 64;                     // head_dim
constexpr int PF_P = 16;                     // tokens per page
constexpr int PF_NST = 4;                    // ring depth (pages in flight per CTA)
constexpr int PF_ROWS = 32;                  // query rows (token, head) per consumer warp
constexpr int PF_BUCKETS = 1024;             // plan: tile-cost buckets (pages, clamped)
constexpr int PF_PAGE = PF_P * PF_D * 8 * 2; // 16 KiB: one page of one layer, K or V, 8 heads
constexpr int PF_STAGE = 2 * PF_PAGE;        // K + V
constexpr int PF_QSTAGE = PF_ROWS * PF_D * 2;  // 4 KiB of query rows per warp

struct PrefillArgs {
  const void* q;
  void* out;
  const int32_t* cu_q;
  const int32_t* kv_lens;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* last_page_len;
  const int2* tiles;
  const int32_t* n_tiles;
  int32_t* st;
  int64_t num_blocks;
  int64_t total_pages;
  int n_seqs, n_tokens, n_heads, layer;
  float scale_log2;
};

// ---------------------------------------------------------------- plan
// Pages a tile [j0, j0 + qt) of a sequence with kv_len keys and q_len queries
// reads: keys up to kv_len - q_len + (last token of the tile). 0 if the
// metadata is inconsistent (the attention kernel flags it).
__device__ __forceinline__ int tile_pages(int64_t kv, int ql, int j0, int qt) {
  if (kv < ql || ql < 1) return 0;
  const int jl = min(j0 + qt, ql) - 1;
  const int64_t c = (kv - ql + jl) / PF_P + 1;
  return int(c < 0x7fffffff ? c : 0x7fffffff);
}

// Decode rows of a mixed batch, for the decode kernel: the q_len == 1
// sequences are listed contiguously (index d), their pages get the decode
// kernel's descriptors {page id, d<<7 | first<<6 | last<<5 | valid, first page
// of d, one past its last page} in listed order, rows[d] = their q / out row,
// rows past the list = -1, *p_dec = pages listed; split-K counters (one per
// listed sequence) zeroed.
struct MixedOut {
  const int32_t* kv_indices;
  const int32_t* kv_lens;
  int64_t total_pages, num_blocks;
  int4* desc;
  int32_t* counters;  // [n_seqs]
  int32_t* rows;      // [n_seqs]
  int64_t* p_dec;
};

__global__ void __launch_bounds__(1024) prefill_plan_kernel(
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ kv_indptr,
    const int32_t* __restrict__ last_page_len, int n_seqs, int n_tokens, int qt, int max_tiles,
    int2* __restrict__ tiles, int32_t* __restrict__ n_tiles, int32_t* st, int mixed, MixedOut mo) {
  __shared__ int cnt[PF_BUCKETS];
  __shared__ int warp_sum[32];
  __shared__ int s_bad, s_total;
  const int tid = threadIdx.x;
  // in a mixed batch the q_len == 1 sequences go to the decode kernel, not into tiles
  const int min_ql = mixed ? 2 : 1;
  for (int b = tid; b < PF_BUCKETS; b += blockDim.x) cnt[b] = 0;
  if (tid == 0) {
    s_bad = (cu_q[0] != 0 || cu_q[n_seqs] != n_tokens) ? 1 : 0;
    s_total = 0;
  }
  __syncthreads();
  auto seq_kv = [&](int s) -> int64_t {
    const int64_t pages = int64_t(kv_indptr[s + 1]) - kv_indptr[s];
    const int lpl = last_page_len[s];
    return (pages >= 1 && lpl >= 1 && lpl <= PF_P) ? (pages - 1) * PF_P + lpl : 0;
  };
  for (int s = tid; s < n_seqs; s += blockDim.x) {
    const int ql = cu_q[s + 1] - cu_q[s];
    if (ql < 0) {
      s_bad = 1;
      continue;
    }
    if (ql < min_ql) continue;
    const int64_t kv = seq_kv(s);
    atomicAdd(&s_total, (ql + qt - 1) / qt);
    for (int j0 = 0; j0 < ql; j0 += qt) atomicAdd(&cnt[min(tile_pages(kv, ql, j0, qt), PF_BUCKETS - 1)], 1);
  }
  __syncthreads();
  if (s_bad || s_total > max_tiles) {
    if (tid == 0) {
      flag(st, PKV_DEV_META_BAD);
      n_tiles[0] = 0;
      n_tiles[1] = n_tiles[2] = 0;  // the lean prefill kernel's item claim and exit counters
      if (mixed) *mo.p_dec = 0;
    }
    __threadfence();  // p_dec is read by the decode kernel before its griddepcontrol.wait
    return;
  }
  // exclusive scan over the buckets from the most expensive down: thread t owns
  // bucket PF_BUCKETS - 1 - t (blockDim.x == PF_BUCKETS)
  const int lane = tid & 31, w = tid >> 5;
  const int mine = cnt[PF_BUCKETS - 1 - tid];
  int incl = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) warp_sum[w] = incl;
  __syncthreads();
  if (w == 0) {
    int x = warp_sum[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += v;
    }
    warp_sum[lane] = x;  // inclusive over warps
  }
  __syncthreads();
  const int start = (w ? warp_sum[w - 1] : 0) + incl - mine;
  __syncthreads();
  cnt[PF_BUCKETS - 1 - tid] = start;
  __syncthreads();
  for (int s = tid; s < n_seqs; s += blockDim.x) {
    const int ql = cu_q[s + 1] - cu_q[s];
    if (ql < min_ql) continue;
    const int64_t kv = seq_kv(s);
    for (int j0 = 0; j0 < ql; j0 += qt) {
      const int pos = atomicAdd(&cnt[min(tile_pages(kv, ql, j0, qt), PF_BUCKETS - 1)], 1);
      tiles[pos] = make_int2(s, j0);
    }
  }
  if (tid == 0) {
    n_tiles[0] = s_total;
    n_tiles[1] = n_tiles[2] = 0;  // the lean prefill kernel's item claim and exit counters
  }
  // the tcgen05 prefill kernel reads the tile list before its griddepcontrol.wait
  // (it starts only once this kernel has completed): stores visible at GPU scope
  __threadfence();
  if (!mixed) return;

  // ---- decode rows of the mixed batch, listed in sequence order
  int base_seq = 0, base_pg = 0;
  for (int c0 = 0; c0 < n_seqs; c0 += blockDim.x) {
    const int s = c0 + tid;
    int isdec = 0, np = 0, lpl = 0;
    int64_t pa = 0;
    if (s < n_seqs && cu_q[s + 1] - cu_q[s] == 1) {
      pa = kv_indptr[s];
      const int64_t pb = kv_indptr[s + 1];
      lpl = last_page_len[s];
      bool bad = pb < pa + 1 || pa < 0 || pb > mo.total_pages || lpl < 1 || lpl > PF_P;
      if (!bad && mo.kv_lens && int64_t(mo.kv_lens[s]) != (pb - pa - 1) * PF_P + lpl) bad = true;
      if (bad) flag(st, PKV_DEV_META_BAD);
      else {
        isdec = 1;
        np = int(pb - pa);
      }
    }
    int tot_seq, tot_pg;
    const int d = base_seq + block_excl_scan(isdec, warp_sum, &tot_seq);
    const int off = base_pg + block_excl_scan(np, warp_sum, &tot_pg);
    if (isdec) {
      mo.rows[d] = cu_q[s];
      mo.counters[d] = 0;
      for (int p = 0; p < np; ++p) {
        const int id = mo.kv_indices[pa + p];
        if (id < 0 || id >= mo.num_blocks) flag(st, PKV_DEV_SLOT_OOB);
        const int first = p == 0, last = p == np - 1;
        mo.desc[off + p] = make_int4(id, (d << 7) | (first << 6) | (last << 5) | (last ? lpl : PF_P), off, off + np);
      }
    }
    base_seq += tot_seq;
    base_pg += tot_pg;
  }
  for (int d = base_seq + tid; d < n_seqs; d += blockDim.x) mo.rows[d] = -1;
  if (tid == 0) *mo.p_dec = base_pg;
  // The decode kernel reads p_dec and the descriptors before its
  // griddepcontrol.wait (it starts only once this kernel has completed, which
  // never triggers its dependents early): the stores are made visible at GPU
  // scope before this block exits.
  __threadfence();
}

// ---------------------------------------------------------------- attention
// bits of a V fragment register (keys k, k + 1 packed low/high) kept when the
// sequence's last page holds `valid` written tokens
__device__ __forceinline__ uint32_t key_keep(int k, int valid) {
  return (k < valid ? 0x0000ffffu : 0u) | (k + 1 < valid ? 0xffff0000u : 0u);
}

template <typename T, int G>
__global__ void __launch_bounds__(512, 1) prefill_kernel(const __grid_constant__ CUtensorMap tmap,
                                                         const PrefillArgs a) {
  constexpr int TPW = PF_ROWS / G;  // tokens per warp
  constexpr int QT = 2 * TPW;       // tokens per tile (two warps per KV head)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nw = blockDim.x >> 5;  // 2 * n_kv_heads consumer warps
  const int n_kv = nw >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  unsigned char* stages = smem;
  unsigned char* qstage = smem + size_t(PF_NST) * PF_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(qstage + size_t(nw) * PF_QSTAGE);
  uint64_t* empty = full + PF_NST;
  __shared__ int s_bad;

  if (int(blockIdx.x) >= *a.n_tiles) return;
  const int2 tile = a.tiles[blockIdx.x];
  const int s = tile.x, j0 = tile.y;
  bool bad = s < 0 || s >= a.n_seqs;
  int q0 = 0, ql = 0, lpl = 0;
  int64_t pa = 0, pb = 0;
  if (!bad) {
    q0 = a.cu_q[s];
    ql = a.cu_q[s + 1] - q0;
    pa = a.kv_indptr[s];
    pb = a.kv_indptr[s + 1];
    lpl = a.last_page_len[s];
  }
  const int64_t npages = pb - pa;
  const int64_t kv64 = (npages - 1) * PF_P + lpl;
  bad = bad || npages < 1 || pa < 0 || pb > a.total_pages || lpl < 1 || lpl > PF_P || ql < 1 ||
        j0 < 0 || j0 >= ql || kv64 < ql || kv64 >= 0x7fffffff || q0 < 0 || q0 + ql > a.n_tokens;
  if (!bad && a.kv_lens && a.kv_lens[s] != kv64) bad = true;
  const int kv = bad ? 0 : int(kv64);
  const int n_pg = bad ? 0 : tile_pages(kv, ql, j0, QT);
  if (threadIdx.x == 0) s_bad = bad ? 1 : 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n_pg; i += blockDim.x) {
    const int id = a.kv_indices[pa + i];
    if (id < 0 || id >= a.num_blocks) s_bad = 2;
  }
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < PF_NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], nw);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int kvh = warp >> 1, half = warp & 1;
  const int tw0 = j0 + half * TPW;  // first (chunk-relative) token of this warp's rows
  T* out = static_cast<T*>(a.out);
  unsigned char* qs = qstage + size_t(warp) * PF_QSTAGE;
  // row r of a warp: query head kvh * G + r / TPW, token tw0 + r % TPW
  auto out_row = [&](int r) -> T* {
    const int j = tw0 + r % TPW;
    return j < ql ? out + ((int64_t(q0) + j) * a.n_heads + kvh * G + r / TPW) * PF_D : nullptr;
  };
  if (s_bad) {
    if (threadIdx.x == 0) flag(a.st, s_bad == 1 ? PKV_DEV_META_BAD : PKV_DEV_SLOT_OOB);
    if (s_bad == 2) {  // rows are known: zero them
      for (int it = 0; it < PF_ROWS * 8 / 32; ++it) {
        const int idx = it * 32 + lane;
        if (T* o = out_row(idx >> 3)) reinterpret_cast<uint4*>(o)[idx & 7] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    return;
  }

  const int kv_coord = 2 * a.layer;
  const uint32_t tx_bytes = 2u * n_kv * PF_P * PF_D * 2;
  int issued = 0;  // thread 0 only
  auto issue = [&](int i) {
    const int slot = i % PF_NST;
    const int id = a.kv_indices[pa + i];
    unsigned char* dst = stages + size_t(slot) * PF_STAGE;
    mbar_arrive_expect_tx(&full[slot], tx_bytes);
    tma_load_4d(dst, &tmap, &full[slot], 0, id * PF_P, 0, kv_coord);
    tma_load_4d(dst + PF_PAGE, &tmap, &full[slot], 0, id * PF_P, 0, kv_coord + 1);
    issued = i + 1;
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(PF_NST, n_pg); ++i) issue(i);

  // this warp's 32 query rows -> shared memory, 128B-swizzled (zeros past q_len)
  {
    const T* qg = static_cast<const T*>(a.q);
#pragma unroll
    for (int it = 0; it < PF_ROWS * 8 / 32; ++it) {
      const int idx = it * 32 + lane;
      const int r = idx >> 3, c = idx & 7;
      const int j = tw0 + r % TPW;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (j < ql)
        v = __ldg(reinterpret_cast<const uint4*>(qg + ((int64_t(q0) + j) * a.n_heads + kvh * G + r / TPW) * PF_D) + c);
      *reinterpret_cast<uint4*>(qs + r * 128 + ((c ^ (r & 7)) << 4)) = v;
    }
    __syncwarp();
  }
  const uint32_t qs_u = smem_u32(qs);

  // last visible key of each of this thread's rows (16 mt + g + 8 e); -1: padding row
  int lim[2][2];
  int lim_min = 0x7fffffff, lim_max = -1;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = tw0 + (16 * mt + g + 8 * e) % TPW;
      lim[mt][e] = j < ql ? kv - ql + j : -1;
      lim_min = min(lim_min, lim[mt][e]);
      lim_max = max(lim_max, lim[mt][e]);
    }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) lim_max = max(lim_max, __shfl_xor_sync(0xffffffffu, lim_max, off));

  float o[2][8][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nd = 0; nd < 8; ++nd)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][nd][e] = 0.f;
  float m[2][2], l[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      m[mt][e] = -INFINITY;
      l[mt][e] = 0.f;
    }

  const int q_row = lane & 15, q_chk = lane >> 4;                     // A: ldmatrix x4
  const int k_row = lane & 7, k_chk = lane >> 3;                      // B = K: x4 over 4 chunks
  const int v_row = (lane & 7) + ((lane >> 3) & 1) * 8, v_chk = lane >> 4;  // B = V: x4.trans
  const float sl2 = a.scale_log2;
  bool dead = false;

  for (int i = 0; i < n_pg; ++i) {
    const int slot = i % PF_NST;
    if (warp == 0) {
      // refill the slot of page i - 1 once every warp has released it
      if (lane == 0 && i >= 1 && !dead && i - 1 + PF_NST < n_pg) {
        if (mbar_wait_bounded(&empty[(i - 1) % PF_NST], ((i - 1) / PF_NST) & 1, a.st)) issue(i - 1 + PF_NST);
        else dead = true;
      }
      __syncwarp();
    }
    if (!dead && !mbar_wait_bounded(&full[slot], (i / PF_NST) & 1, a.st)) dead = true;
    dead = __any_sync(0xffffffffu, dead);
    if (!dead && PF_P * i <= lim_max) {
      const uint32_t kbase = smem_u32(stages + size_t(slot) * PF_STAGE) + kvh * (PF_P * 128);
      const uint32_t vbase = kbase + PF_PAGE;
      // S[32 rows x 16 keys] = Q . K^T
      float sc[2][2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[mt][nt][e] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t kf[2][4];  // [nt][chunk 4kp + j]
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int key = 8 * nt + k_row, chunk = 4 * kp + k_chk;
          ldsm_x4(kf[nt][0], kf[nt][1], kf[nt][2], kf[nt][3], kbase + key * 128 + ((chunk ^ (key & 7)) << 4));
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int ks = 2 * kp + kk;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            uint32_t qa[4];
            const int row = 16 * mt + q_row, chunk = 2 * ks + q_chk;
            ldsm_x4(qa[0], qa[1], qa[2], qa[3], qs_u + row * 128 + ((chunk ^ (row & 7)) << 4));
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) MmaOp<T>::run(sc[mt][nt], qa, kf[nt][2 * kk], kf[nt][2 * kk + 1]);
          }
        }
      }
      // scale (log2 domain), causal mask, online softmax
      const int kb0 = PF_P * i;
      const bool tail = kb0 + PF_P - 1 > lim_min;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kb0 + 8 * nt + 2 * c4 + (e & 1);
            const float x = sc[mt][nt][e] * sl2;
            sc[mt][nt][e] = (tail && key > lim[mt][e >> 1]) ? -INFINITY : x;
          }
      uint32_t pf[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float mx = fmaxf(fmaxf(sc[mt][0][2 * e], sc[mt][0][2 * e + 1]),
                           fmaxf(sc[mt][1][2 * e], sc[mt][1][2 * e + 1]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float mn = fmaxf(m[mt][e], mx);
          const float base = mn == -INFINITY ? 0.f : mn;
          const float al = ex2(m[mt][e] - base);
          m[mt][e] = mn;
          float ls = 0.f;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            sc[mt][nt][2 * e] = ex2(sc[mt][nt][2 * e] - base);
            sc[mt][nt][2 * e + 1] = ex2(sc[mt][nt][2 * e + 1] - base);
            ls += sc[mt][nt][2 * e] + sc[mt][nt][2 * e + 1];
          }
          l[mt][e] = l[mt][e] * al + ls;
#pragma unroll
          for (int nd = 0; nd < 8; ++nd) {
            o[mt][nd][2 * e] *= al;
            o[mt][nd][2 * e + 1] *= al;
          }
        }
        pf[mt][0] = MmaOp<T>::pack(sc[mt][0][0], sc[mt][0][1]);
        pf[mt][1] = MmaOp<T>::pack(sc[mt][0][2], sc[mt][0][3]);
        pf[mt][2] = MmaOp<T>::pack(sc[mt][1][0], sc[mt][1][1]);
        pf[mt][3] = MmaOp<T>::pack(sc[mt][1][2], sc[mt][1][3]);
      }
      // O[32 rows x 64 dims] += P[32 x 16] . V[16 x 64]
      const bool vtail = (i == npages - 1) && lpl < PF_P;
      const uint32_t keep_lo = vtail ? key_keep(2 * c4, lpl) : 0xffffffffu;
      const uint32_t keep_hi = vtail ? key_keep(8 + 2 * c4, lpl) : 0xffffffffu;
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t vf[4];
        const int chunk = 2 * dp + v_chk;
        ldsm_x4_t(vf[0], vf[1], vf[2], vf[3], vbase + v_row * 128 + ((chunk ^ (v_row & 7)) << 4));
        vf[0] &= keep_lo;
        vf[1] &= keep_hi;
        vf[2] &= keep_lo;
        vf[3] &= keep_hi;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          MmaOp<T>::run(o[mt][2 * dp], pf[mt], vf[0], vf[1]);
          MmaOp<T>::run(o[mt][2 * dp + 1], pf[mt], vf[2], vf[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[slot])) : "memory");
  }

  // epilogue: O / l -> this warp's (now free) query staging -> 16-byte row stores
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float lt = l[mt][e];
      lt += __shfl_xor_sync(0xffffffffu, lt, 1);
      lt += __shfl_xor_sync(0xffffffffu, lt, 2);
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const int r = 16 * mt + g + 8 * e;
#pragma unroll
      for (int nd = 0; nd < 8; ++nd)
        *reinterpret_cast<uint32_t*>(qs + r * 128 + ((nd ^ (r & 7)) << 4) + c4 * 4) =
            MmaOp<T>::pack(o[mt][nd][2 * e] * inv, o[mt][nd][2 * e + 1] * inv);
    }
  __syncwarp();
#pragma unroll
  for (int it = 0; it < PF_ROWS * 8 / 32; ++it) {
    const int idx = it * 32 + lane;
    const int r = idx >> 3, c = idx & 7;
    if (T* orow = out_row(r)) reinterpret_cast<uint4*>(orow)[c] = *reinterpret_cast<const uint4*>(qs + r * 128 + ((c ^ (r & 7)) << 4));
  }
  // error path only: let this CTA's own copies land before its shared memory is released
  if (threadIdx.x == 0 && dead) {
    for (int i = max(0, issued - PF_NST); i < issued; ++i)
      mbar_wait_bounded(&full[i % PF_NST], (i / PF_NST) & 1, nullptr);
  }
}

size_t prefill_smem(int n_kv) {
  return 1024 + size_t(PF_NST) * PF_STAGE + size_t(2 * n_kv) * PF_QSTAGE + 2 * PF_NST * 8;
}

template <typename T, int G>
int launch_prefill_t(const pkv_pool& p, const CUtensorMap& tm, const PrefillArgs& a, int grid,
                     cudaStream_t s) {
  static std::mutex mu;
  static std::vector<char> ready;
  int dev = 0;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  const size_t smem = prefill_smem(8);
  {
    std::lock_guard<std::mutex> lock(mu);
    if ((int)ready.size() <= dev) ready.resize(dev + 1, 0);
    if (!ready[dev]) {
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_kernel<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      ready[dev] = 1;
    }
  }
  prefill_kernel<T, G><<<grid, 64 * p.n_kv_heads, prefill_smem(p.n_kv_heads), s>>>(tm, a);
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

template <typename T>
int launch_prefill_g(const pkv_pool& p, int groups, const CUtensorMap& tm, const PrefillArgs& a,
                     int grid, cudaStream_t s) {
  switch (groups) {
    case 1: return launch_prefill_t<T, 1>(p, tm, a, grid, s);
    case 2: return launch_prefill_t<T, 2>(p, tm, a, grid, s);
    case 4: return launch_prefill_t<T, 4>(p, tm, a, grid, s);
    case 8: return launch_prefill_t<T, 8>(p, tm, a, grid, s);
  }
  return fail(PKV_ERR_UNSUPPORTED, "prefill kernel: unsupported GQA group size");
}

}  // namespace

bool prefill_supported(const pkv_pool& p, int n_heads) {
  if (p.dtype != PKV_F16 && p.dtype != PKV_BF16) return false;
  if (p.head_dim != PF_D || p.block_size != PF_P) return false;
  if (p.n_kv_heads < 1 || p.n_kv_heads > 8) return false;
  if (n_heads % p.n_kv_heads) return false;
  const int gq = n_heads / p.n_kv_heads;
  return gq == 1 || gq == 2 || gq == 4 || gq == 8;
}

// The tcgen05 kernel (pkv_prefill_tc.cu) is the default; PKV_PREFILL_TC=0 selects
// this file's mma.sync kernel (for comparisons). Read at every plan and every
// launch, so it must not change between a step's plan and its attends.
bool prefill_use_tc() {
  const char* e = getenv("PKV_PREFILL_TC");
  return !(e && e[0] == '0');
}

int prefill_tile_tokens(int n_heads, int n_kv_heads) {
  if (prefill_use_tc()) return prefill_tc_tile_tokens(n_heads, n_kv_heads);
  return 2 * (PF_ROWS / (n_heads / n_kv_heads));
}

int64_t prefill_tiles_cap(int n_seqs, int64_t total_pages) {
  // tiles <= n_tokens / QT + n_seqs with QT >= 8 and n_tokens <= 16 * total_pages
  return 2 * std::max<int64_t>(total_pages, 1) + n_seqs;
}

int prefill_plan(const pkv_pool& p, int n_heads, const pkv_batch& b, int2* tiles, int32_t* n_tiles,
                 int64_t tiles_cap, const PrefillMixedPlan* mixed, cudaStream_t s) {
  const int qt = prefill_tile_tokens(n_heads, p.n_kv_heads);
  const int cap = int(std::min<int64_t>(tiles_cap, 0x7fffffff));
  MixedOut mo{};
  if (mixed) {
    mo.kv_indices = b.kv_indices;
    mo.kv_lens = b.kv_lens;
    mo.total_pages = b.total_pages;
    mo.num_blocks = p.num_blocks;
    mo.desc = mixed->desc;
    mo.counters = mixed->counters;
    mo.rows = mixed->rows;
    mo.p_dec = mixed->p_dec;
  }
  prefill_plan_kernel<<<1, PF_BUCKETS, 0, s>>>(b.cu_query_lens, b.kv_indptr, b.kv_last_page_len,
                                               b.n_seqs, b.n_tokens, qt, cap, tiles, n_tiles,
                                               b.dev_status, mixed ? 1 : 0, mo);
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

int prefill_attend(const pkv_pool& p, int layer, int n_heads, const void* q, void* out, float scale,
                   const pkv_batch& b, const int2* tiles, const int32_t* n_tiles, int64_t tiles_cap,
                   cudaStream_t s) {
  if (prefill_use_tc()) return prefill_tc_attend(p, layer, n_heads, q, out, scale, b, tiles, n_tiles, tiles_cap, s);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
  CUtensorMap tm;
  if (int rc = pool_tmap(p, &tm)) return rc;
  PrefillArgs a;
  a.q = q;
  a.out = out;
  a.cu_q = b.cu_query_lens;
  a.kv_lens = b.kv_lens;
  a.kv_indptr = b.kv_indptr;
  a.kv_indices = b.kv_indices;
  a.last_page_len = b.kv_last_page_len;
  a.tiles = tiles;
  a.n_tiles = n_tiles;
  a.st = b.dev_status;
  a.num_blocks = p.num_blocks;
  a.total_pages = b.total_pages;
  a.n_seqs = b.n_seqs;
  a.n_tokens = b.n_tokens;
  a.n_heads = n_heads;
  a.layer = layer;
  a.scale_log2 = scale * 1.4426950408889634f;
  const int qt = prefill_tile_tokens(n_heads, p.n_kv_heads);
  const int64_t bound = (int64_t(b.n_tokens) + qt - 1) / qt + b.n_seqs;
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(bound, std::min<int64_t>(tiles_cap, 0x7fffffff))));
  const int groups = n_heads / p.n_kv_heads;
  if (p.dtype == PKV_F16) return launch_prefill_g<__half>(p, groups, tm, a, grid, s);
  return launch_prefill_g<__nv_bfloat16>(p, groups, tm, a, grid, s);
}

}  // namespace pkv
