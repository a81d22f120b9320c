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
//                   Sequences cut by a range boundary are merged by the last
//                   CTA to finish (atomic counter, no waiting).
//   generic_kernel  any geometry / dtype / query length (chunked prefill,
//                   mixed batches): one warp per (token, query head), CUDA cores.
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
constexpr int DK_MERGE_CHUNK = 16;         // split-K pieces merged per pass
constexpr int DK_MERGE_HEADS = 64;         // query heads of the decode kernel (n_heads <= 64)
constexpr int DK_MERGE_PER = 8;            // merged outputs per consumer thread per pass

// ---------------------------------------------------------------- workspace
struct WsLayout {
  size_t page_desc = 0;  // int2[total_pages]
  size_t counters = 0;   // int32[n_seqs]
  size_t partial = 0;    // float[2 * grid][n_heads][D + 2]
  size_t total = 0;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

WsLayout ws_layout(int n_heads, int n_seqs, int64_t total_pages, int max_grid, int head_dim) {
  WsLayout w;
  size_t off = 0;
  w.page_desc = off;
  off = align256(off + sizeof(int2) * size_t(std::max<int64_t>(total_pages, 1)));
  w.counters = off;
  off = align256(off + sizeof(int32_t) * size_t(std::max(n_seqs, 1)));
  w.partial = off;
  off = align256(off + sizeof(float) * size_t(2) * max_grid * n_heads * (head_dim + 2));
  w.total = off;
  return w;
}

// ---------------------------------------------------------------- plan
// page_desc[p] = {page id, (seq << 7) | (first << 6) | (last << 5) | valid}
__global__ void plan_kernel(const int32_t* __restrict__ kv_indptr,
                            const int32_t* __restrict__ kv_indices,
                            const int32_t* __restrict__ last_page_len,
                            const int32_t* __restrict__ kv_lens,
                            const int32_t* __restrict__ cu_q, int n_seqs, int64_t total_pages,
                            int block_size, int64_t num_blocks, int2* __restrict__ desc,
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
    return;
  }
  for (int64_t p = a + lane; p < b; p += 32) {
    const int id = kv_indices[p];
    if (id < 0 || id >= num_blocks) flag(st, PKV_DEV_SLOT_OOB);
    const int first = (p == a), last = (p == b - 1);
    const int valid = last ? lpl : block_size;
    desc[p] = make_int2(id, (s << 7) | (first << 6) | (last << 5) | valid);
  }
}

// ---------------------------------------------------------------- decode
struct DecodeArgs {
  const void* q;
  void* out;
  const int32_t* kv_indptr;
  const int2* desc;
  float* partial;
  int32_t* counters;
  int32_t* st;
  int64_t total_pages;
  int n_seqs;
  int n_heads;
  int layer;
  float scale_log2;
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

// One CTA = one producer warp + one consumer warp per KV head. The producer
// streams whole pages: one TMA box per page for K and one for V, each the full
// contiguous 16 KiB [16 tok][8 heads][64] page, read through a permuted view of
// the pool (dims D, T, H) so that it lands in shared memory as [head][tok][64]
// with the 128B swizzle keyed on the token (conflict-free ldmatrix for a head's
// 16 tokens). Consumer warp h reads its head's 2 KiB slice of each stage.
template <typename T, int GROUPS, int NST, int MINB>
__global__ void __launch_bounds__(288, MINB) decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                           const DecodeArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_cons = (blockDim.x >> 5) - 1;  // consumer warps == KV heads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  constexpr int PAGE = DK_P * DK_D * 8 * 2;  // 16 KiB: one page of one layer, K or V (8 heads)
  constexpr int STAGE = 2 * PAGE;
  unsigned char* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(NST) * STAGE);
  uint64_t* empty = full + NST;
  T* ostage_all = reinterpret_cast<T*>(smem + size_t(NST) * STAGE + bar_bytes(2, NST));
  __shared__ int s_last;
  // merge scratch: per-head running max / normaliser / carry and per-piece weights
  __shared__ float s_mrg_m[DK_MERGE_HEADS], s_mrg_W[DK_MERGE_HEADS], s_mrg_scale[DK_MERGE_HEADS];
  __shared__ float s_mrg_w[DK_MERGE_CHUNK * DK_MERGE_HEADS];
  __shared__ float s_mrg_acc[DK_MERGE_HEADS * DK_D];

  const int64_t P = a.total_pages;
  const int G = gridDim.x;
  const int c = blockIdx.x;
  const int64_t p0 = int64_t(c) * P / G, p1 = int64_t(c + 1) * P / G;
  if (p0 >= p1) return;
  const int R = int(p1 - p0);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], n_cons);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // page descriptors: lane j holds window entries [wb + j] (cur) and [wb + 32 + j] (nxt)
  int wb = 0;
  int2 dcur = make_int2(-1, -1), dnxt = make_int2(-1, -1);
  if (lane < R) dcur = a.desc[p0 + lane];
  if (32 + lane < R) dnxt = a.desc[p0 + 32 + lane];
  auto desc_at = [&](int i) -> int2 {  // uniform i in [wb, wb + 64)
    const bool in_cur = i < wb + 32;
    int2 d;
    d.x = __shfl_sync(0xffffffffu, in_cur ? dcur.x : dnxt.x, i & 31);
    d.y = __shfl_sync(0xffffffffu, in_cur ? dcur.y : dnxt.y, i & 31);
    return d;
  };
  auto slide = [&](int i) {
    if (i == wb + 32) {
      wb += 32;
      dcur = dnxt;
      dnxt = make_int2(-1, -1);
      if (wb + 32 + lane < R) dnxt = a.desc[p0 + wb + 32 + lane];
    }
  };
  const int kv_coord = 2 * a.layer;

  if (warp == n_cons) {
    // ---------------- producer warp
    bool dead = false;
    for (int i = 0; i < R; ++i) {
      slide(i);
      const int2 d = desc_at(i);
      const int st = i % NST;
      if (lane == 0 && !dead) {
        if (i >= NST && !mbar_wait_bounded(&empty[st], ((i / NST) - 1) & 1, a.st)) dead = true;
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
  T* ostage = ostage_all + size_t(h) * GROUPS * DK_D;
  const int n_cons_threads = n_cons * 32;
  auto cons_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"r"(n_cons_threads) : "memory"); };

  uint32_t qb[4][2], qn[4][2];
  float o[4][4];
  float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
  int cur_seq = -1, nxt_seq = -1;
  bool seen_first = false, dead = false;
  int64_t seq_fa = 0, seq_fb = 0;
  const int first_seq = desc_at(0).y >> 7;

  const int k_tok = (lane & 7) + ((lane >> 3) & 1) * 8, k_chk = lane >> 4;
  const int v_tok = (lane & 7) + (lane >> 4) * 8, v_chk = (lane >> 3) & 1;

  for (int i = 0; i < R; ++i) {
    slide(i);
    const int2 d = desc_at(i);
    const int seq = d.y >> 7;
    const bool is_first = (d.y >> 6) & 1, is_last = (d.y >> 5) & 1;
    const int valid = d.y & 31;
    const int st = i % NST;
    unsigned char* kt = stages + size_t(st) * STAGE + h * (DK_P * DK_D * 2);
    unsigned char* vt = kt + PAGE;
    if (!dead && !mbar_wait_bounded(&full[st], (i / NST) & 1, a.st)) dead = true;

    if (seq < 0 || seq >= a.n_seqs || valid < 1 || valid > DK_P) {
      // a page of a sequence the plan rejected: release the stage, compute nothing
      if (lane == 0 && !dead) flag(a.st, PKV_DEV_META_BAD);
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
      continue;
    }
    if (seq != cur_seq) {
      if (seq == nxt_seq) {
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) { qb[ks][0] = qn[ks][0]; qb[ks][1] = qn[ks][1]; }
      } else {
        load_q_frag<T, GROUPS>(q, seq, a.n_heads, h, g, c4, qb);
      }
      cur_seq = seq;
      nxt_seq = seq + 1;
      seq_fa = a.kv_indptr[seq];  // needed only if the sequence ends split
      seq_fb = a.kv_indptr[seq + 1];
      if (nxt_seq < a.n_seqs) load_q_frag<T, GROUPS>(q, nxt_seq, a.n_heads, h, g, c4, qn);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
      m0 = m1 = -1e30f;
      l0 = l1 = 0.f;
      seen_first = is_first;
    }

    const bool zeroed = valid < DK_P;
    if (zeroed) {  // never let the unwritten tail of a last page reach P.V
      for (int r = valid * 8 + lane; r < DK_P * 8; r += 32)
        reinterpret_cast<uint4*>(vt)[r] = make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
    }

    // S^T[16 tok x 8 heads] = K[16 x 64] . Q^T[64 x 8]
    float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kbase = smem_u32(kt);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {  // two accumulators halve the dependent mma chain
      uint32_t af[4];
      const int chunk = 2 * ks + k_chk;
      ldsm_x4(af[0], af[1], af[2], af[3], kbase + k_tok * 128 + ((chunk ^ (k_tok & 7)) << 4));
      MmaOp<T>::run((ks & 1) ? s2 : s, af, qb[ks][0], qb[ks][1]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] += s2[e];
    // rows g and g+8 are tokens; columns 2*c4, 2*c4+1 are heads of the group
    const bool v0 = g < valid, v1 = (g + 8) < valid;
    s[0] = v0 ? s[0] * a.scale_log2 : -INFINITY;
    s[1] = v0 ? s[1] * a.scale_log2 : -INFINITY;
    s[2] = v1 ? s[2] * a.scale_log2 : -INFINITY;
    s[3] = v1 ? s[3] * a.scale_log2 : -INFINITY;
    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = ex2(m0 - mn0), al1 = ex2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float p00 = ex2(s[0] - mn0), p01 = ex2(s[1] - mn1);
    const float p10 = ex2(s[2] - mn0), p11 = ex2(s[3] - mn1);
    l0 = l0 * al0 + p00 + p10;
    l1 = l1 * al1 + p01 + p11;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      o[mt][0] *= al0;
      o[mt][2] *= al0;
      o[mt][1] *= al1;
      o[mt][3] *= al1;
    }
    const uint32_t pb0 = movmatrix_t(MmaOp<T>::pack(p00, p01));
    const uint32_t pb1 = movmatrix_t(MmaOp<T>::pack(p10, p11));
    // O^T[64 dims x 8 heads] += V^T[64 x 16] . P^T[16 x 8]
    const uint32_t vbase = smem_u32(vt);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t af[4];
      const int chunk = 2 * mt + v_chk;
      ldsm_x4_t(af[0], af[1], af[2], af[3], vbase + v_tok * 128 + ((chunk ^ (v_tok & 7)) << 4));
      MmaOp<T>::run(o[mt], af, pb0, pb1);
    }
    __syncwarp();
    if (lane == 0) {  // release the stage to the producer
      if (zeroed) fence_proxy_async_smem();  // the next TMA must land after the zero stores
      asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
    }

    // end of this sequence within the CTA's range?
    const bool seq_ends = is_last || (i == R - 1);
    if (!seq_ends) continue;
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
    }
    const int j0 = 2 * c4, j1 = 2 * c4 + 1;
    if (seen_first && is_last) {
      // the whole sequence lives in this CTA: normalise and store
      const float i0 = 1.f / lt0, i1 = 1.f / lt1;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int d0 = mt * 16 + g, d1 = d0 + 8;
        if (j0 < GROUPS) {
          ostage[j0 * DK_D + d0] = from_f<T>(o[mt][0] * i0);
          ostage[j0 * DK_D + d1] = from_f<T>(o[mt][2] * i0);
        }
        if (j1 < GROUPS) {
          ostage[j1 * DK_D + d0] = from_f<T>(o[mt][1] * i1);
          ostage[j1 * DK_D + d1] = from_f<T>(o[mt][3] * i1);
        }
      }
      __syncwarp();
      uint4* dst = reinterpret_cast<uint4*>(out + (int64_t(seq) * a.n_heads + h * GROUPS) * DK_D);
      for (int ch = lane; ch < GROUPS * 8; ch += 32) dst[ch] = reinterpret_cast<const uint4*>(ostage)[ch];
      __syncwarp();
    } else {
      // a piece of a sequence cut by a range boundary: write (m, l, O/l)
      const int slot = (seq == first_seq) ? 0 : 1;
      float* pb = a.partial + (size_t(2 * c + slot) * a.n_heads + h * GROUPS) * (DK_D + 2);
      const float i0 = 1.f / lt0, i1 = 1.f / lt1;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int d0 = mt * 16 + g, d1 = d0 + 8;
        if (j0 < GROUPS) {
          pb[j0 * (DK_D + 2) + d0] = o[mt][0] * i0;
          pb[j0 * (DK_D + 2) + d1] = o[mt][2] * i0;
        }
        if (j1 < GROUPS) {
          pb[j1 * (DK_D + 2) + d0] = o[mt][1] * i1;
          pb[j1 * (DK_D + 2) + d1] = o[mt][3] * i1;
        }
      }
      if (g == 0) {
        if (j0 < GROUPS) { pb[j0 * (DK_D + 2) + DK_D] = m0; pb[j0 * (DK_D + 2) + DK_D + 1] = lt0; }
        if (j1 < GROUPS) { pb[j1 * (DK_D + 2) + DK_D] = m1; pb[j1 * (DK_D + 2) + DK_D + 1] = lt1; }
      }
      cons_sync();  // every consumer warp's piece is written
      const int64_t fa = seq_fa, fb = seq_fb;
      const int cf = cta_of(fa, P, G), cl = cta_of(fb - 1, P, G);
      if (threadIdx.x == 0) {
        // one acq_rel RMW at gpu scope: releases this CTA's piece (cumulative
        // over the barrier above) and, for the last CTA, acquires the others'
        int prev;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                     : "=r"(prev) : "l"(a.counters + seq) : "memory");
        s_last = (prev == cl - cf);
      }
      cons_sync();
      if (s_last) {
        // merge the pieces: per-head weights first (one pass over (m, l)),
        // then every output element as one independent sweep over the pieces
        const int nh = a.n_heads;
        const int npieces = cl - cf + 1;
        for (int p0m = 0; p0m < npieces; p0m += DK_MERGE_CHUNK) {
          const int np = min(DK_MERGE_CHUNK, npieces - p0m);
          for (int t = threadIdx.x; t < nh; t += n_cons_threads) {
            float M = -1e30f;
            for (int k = 0; k < np; ++k) {
              const int cc = cf + p0m + k;
              const int sl = (cc == cf && fa > int64_t(cc) * P / G) ? 1 : 0;
              M = fmaxf(M, __ldcg(a.partial + (size_t(2 * cc + sl) * nh + t) * (DK_D + 2) + DK_D));
            }
            if (p0m > 0) M = fmaxf(M, s_mrg_m[t]);
            float W = 0.f;
            for (int k = 0; k < np; ++k) {
              const int cc = cf + p0m + k;
              const int sl = (cc == cf && fa > int64_t(cc) * P / G) ? 1 : 0;
              const float* pp = a.partial + (size_t(2 * cc + sl) * nh + t) * (DK_D + 2);
              const float w = __ldcg(pp + DK_D + 1) * ex2(__ldcg(pp + DK_D) - M);
              s_mrg_w[k * DK_MERGE_HEADS + t] = w;
              W += w;
            }
            // rescale what earlier chunks accumulated to this chunk's max
            const float carry = (p0m > 0) ? ex2(s_mrg_m[t] - M) : 0.f;
            s_mrg_scale[t] = carry;
            s_mrg_W[t] = (p0m > 0 ? s_mrg_W[t] * carry : 0.f) + W;
            s_mrg_m[t] = M;
          }
          cons_sync();
          // every thread owns DK_MERGE_PER outputs; all their loads are issued
          // before any is consumed (one L2 round trip per pass, not one per output)
          for (int base = 0; base < nh * DK_D; base += n_cons_threads * DK_MERGE_PER) {
            float acc[DK_MERGE_PER];
#pragma unroll
            for (int r = 0; r < DK_MERGE_PER; ++r) {
              const int idx = base + r * n_cons_threads + threadIdx.x;
              acc[r] = (p0m > 0 && idx < nh * DK_D) ? s_mrg_acc[idx] * s_mrg_scale[idx / DK_D] : 0.f;
            }
            for (int k = 0; k < np; ++k) {
              const int cc = cf + p0m + k;
              const int sl = (cc == cf && fa > int64_t(cc) * P / G) ? 1 : 0;
              const float* pp = a.partial + size_t(2 * cc + sl) * nh * (DK_D + 2);
              float v[DK_MERGE_PER];
#pragma unroll
              for (int r = 0; r < DK_MERGE_PER; ++r) {
                const int idx = base + r * n_cons_threads + threadIdx.x;
                v[r] = idx < nh * DK_D ? __ldcg(pp + (idx / DK_D) * (DK_D + 2) + idx % DK_D) : 0.f;
              }
#pragma unroll
              for (int r = 0; r < DK_MERGE_PER; ++r) {
                const int idx = base + r * n_cons_threads + threadIdx.x;
                if (idx < nh * DK_D) acc[r] += s_mrg_w[k * DK_MERGE_HEADS + idx / DK_D] * v[r];
              }
            }
#pragma unroll
            for (int r = 0; r < DK_MERGE_PER; ++r) {
              const int idx = base + r * n_cons_threads + threadIdx.x;
              if (idx >= nh * DK_D) continue;
              const int hh = idx / DK_D, dd = idx % DK_D;
              if (p0m + np < npieces) s_mrg_acc[idx] = acc[r];
              else out[(int64_t(seq) * nh + hh) * DK_D + dd] = from_f<T>(acc[r] / s_mrg_W[hh]);
            }
          }
          cons_sync();
        }
        if (threadIdx.x == 0) a.counters[seq] = 0;
      }
    }
  }
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
  int num_layers, block_size, n_kv_heads, head_dim, dtype;
  CUtensorMap map;
};

int get_tmap(const pkv_pool& p, CUtensorMap* out) {
  static std::mutex mu;
  static std::vector<TmapEntry> cache;
  int dev = 0;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : cache) {
    if (e.device == dev && e.base == p.base && e.num_blocks == p.num_blocks &&
        e.num_layers == p.num_layers && e.block_size == p.block_size &&
        e.n_kv_heads == p.n_kv_heads && e.head_dim == p.head_dim && e.dtype == p.dtype) {
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
  TmapEntry e{dev, p.base, p.num_blocks, p.num_layers, p.block_size, p.n_kv_heads, p.head_dim, p.dtype, {}};
  // Permuted view of the pool: dims (D, token slot, KV head, layer*2+kv) with
  // strides (elem, row, head_dim*elem, slab). One box = one whole page of one
  // layer's K or V, landing in shared memory as [head][token][D].
  const cuuint64_t dims[4] = {cuuint64_t(p.head_dim), cuuint64_t(p.num_blocks) * p.block_size,
                              cuuint64_t(p.n_kv_heads), cuuint64_t(2) * p.num_layers};
  const cuuint64_t strides[3] = {cuuint64_t(row_bytes(p)), cuuint64_t(p.head_dim) * es,
                                 cuuint64_t(slab_bytes(p))};
  const cuuint32_t box[4] = {cuuint32_t(p.head_dim), cuuint32_t(p.block_size),
                             cuuint32_t(p.n_kv_heads), 1u};
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
  return 1024 + nst * stage + bar_bytes(2, nst) + size_t(n_kv_heads) * groups * DK_D * 2;
}

// Ring depth and CTAs per SM of the decode kernel. Defaults are the tuned
// values; PKV_DECODE_NST (2, 3, 4 or 6) and PKV_DECODE_CTAS_PER_SM override them
// for launch-shape sweeps.
int decode_nst() {
  static int v = [] {
    const char* e = getenv("PKV_DECODE_NST");
    const int n = e ? atoi(e) : DK_NST;
    return (n == 2 || n == 3 || n == 4 || n == 6) ? n : DK_NST;
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
template <typename T, int GROUPS, int NST, int MINB>
int decode_grid_limit(int n_kv_heads) {
  static std::mutex mu;
  static std::vector<std::array<int, 9>> occ;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)occ.size() <= dev) occ.resize(dev + 1, std::array<int, 9>{});
  int& o = occ[dev][n_kv_heads];
  if (!o) {
    auto fn = decode_kernel<T, GROUPS, NST, MINB>;
    const size_t sm = decode_smem(n_kv_heads, GROUPS, NST);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    int v = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, fn, 32 * (n_kv_heads + 1), sm);
    if (e != cudaSuccess) {
      cuda_fail(e, "decode kernel occupancy query");
      return -1;
    }
    o = std::max(1, std::min(v, decode_ctas_per_sm_cap()));
  }
  return o * num_sms();
}

int max_decode_grid() { return num_sms() * 8; }

template <typename T, int GROUPS, int NST, int MINB>
int launch_decode_t(const pkv_pool& p, const CUtensorMap& tm, DecodeArgs& a, int64_t total_pages,
                    cudaStream_t s) {
  int limit = decode_grid_limit<T, GROUPS, NST, MINB>(p.n_kv_heads);
  if (limit <= 0) return PKV_ERR_CUDA;  // message already set
  limit = std::min(limit, max_decode_grid());
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(limit, total_pages)));
  decode_kernel<T, GROUPS, NST, MINB>
      <<<grid, 32 * (p.n_kv_heads + 1), decode_smem(p.n_kv_heads, GROUPS, NST), s>>>(tm, a);
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

template <typename T, int GROUPS>
int launch_decode_n(const pkv_pool& p, const CUtensorMap& tm, DecodeArgs& a, int64_t tp,
                    cudaStream_t s) {
  switch (decode_nst()) {
    case 2: return launch_decode_t<T, GROUPS, 2, 2>(p, tm, a, tp, s);
    case 3: return launch_decode_t<T, GROUPS, 3, 2>(p, tm, a, tp, s);
    case 4: return launch_decode_t<T, GROUPS, 4, 1>(p, tm, a, tp, s);
    default: return launch_decode_t<T, GROUPS, 6, 1>(p, tm, a, tp, s);
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

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" size_t pkv_attend_workspace_size(const pkv_pool* pool, int32_t n_heads, int32_t n_seqs,
                                            int64_t total_pages, int32_t decode_hint) {
  (void)decode_hint;
  const int d = pool ? pool->head_dim : DK_D;
  return ws_layout(n_heads, n_seqs, total_pages, max_decode_grid(), d).total;
}

extern "C" int pkv_plan(const pkv_pool* pool, int32_t n_heads, const pkv_batch* batch,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_pool(pool)) return rc;
  if (int rc = check_batch(*pool, n_heads, batch)) return rc;
  const WsLayout w = ws_layout(n_heads, batch->n_seqs, batch->total_pages, max_decode_grid(), pool->head_dim);
  if (!workspace || workspace_bytes < w.total)
    return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
  char* ws = static_cast<char*>(workspace);
  // every descriptor starts as "no sequence" (-1): pages of a sequence the
  // plan rejects are skipped by the decode kernel instead of read as garbage
  PKV_CUDA_RET(cudaMemsetAsync(ws + w.page_desc, 0xff, sizeof(int2) * size_t(batch->total_pages),
                               static_cast<cudaStream_t>(stream)));
  const int threads = 256;
  const int64_t n_threads = int64_t(batch->n_seqs) * 32;
  plan_kernel<<<unsigned((n_threads + threads - 1) / threads), threads, 0,
                static_cast<cudaStream_t>(stream)>>>(
      batch->kv_indptr, batch->kv_indices, batch->kv_last_page_len, batch->kv_lens,
      batch->cu_query_lens, batch->n_seqs, batch->total_pages, pool->block_size, pool->num_blocks,
      reinterpret_cast<int2*>(ws + w.page_desc), reinterpret_cast<int32_t*>(ws + w.counters),
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

  if (decode_hint && decode_supported(p, n_heads)) {
    if (batch->n_tokens != batch->n_seqs)
      return fail(PKV_ERR_ARG, "decode: n_tokens must equal n_seqs (one query per sequence)");
    if (batch->total_pages == 0) return fail(PKV_ERR_ARG, "decode: empty page table");
    const WsLayout w = ws_layout(n_heads, batch->n_seqs, batch->total_pages, max_decode_grid(), p.head_dim);
    if (!workspace || workspace_bytes < w.total)
      return fail(PKV_ERR_ARG, "workspace too small: need " + std::to_string(w.total) + " bytes");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
      return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
    CUtensorMap tm;
    if (int rc = get_tmap(p, &tm)) return rc;
    char* ws = static_cast<char*>(workspace);
    DecodeArgs a;
    a.q = q;
    a.out = out;
    a.kv_indptr = batch->kv_indptr;
    a.desc = reinterpret_cast<const int2*>(ws + w.page_desc);
    a.partial = reinterpret_cast<float*>(ws + w.partial);
    a.counters = reinterpret_cast<int32_t*>(ws + w.counters);
    a.st = batch->dev_status;
    a.total_pages = batch->total_pages;
    a.n_seqs = batch->n_seqs;
    a.n_heads = n_heads;
    a.layer = layer;
    a.scale_log2 = scale * 1.4426950408889634f;
    const int groups = n_heads / p.n_kv_heads;
    if (p.dtype == PKV_F16) return launch_decode_g<__half>(p, groups, tm, a, batch->total_pages, s);
    return launch_decode_g<__nv_bfloat16>(p, groups, tm, a, batch->total_pages, s);
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

extern "C" int pkv_attend(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* q,
                          void* out, float scale, const pkv_batch* batch, int32_t decode_hint,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (decode_hint && pool && decode_supported(*pool, n_heads)) {
    if (int rc = pkv_plan(pool, n_heads, batch, workspace, workspace_bytes, stream)) return rc;
  }
  return pkv_attend_planned(pool, layer, n_heads, q, out, scale, batch, decode_hint, workspace,
                            workspace_bytes, stream);
}
