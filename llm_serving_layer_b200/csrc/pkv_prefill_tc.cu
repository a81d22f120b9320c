// pkv_prefill_tc.cu — chunked-prefill / mixed-batch attention on the
// 5th-generation tensor cores: tcgen05 MMAs with their accumulators in tensor
// memory (TMEM), operands staged in shared memory by TMA.
//
// Work item = one tile of query rows of one sequence for ONE KV head: 128 rows =
// TPT = 128 / G tokens x the G query heads that share the KV head. The kernels
// share the roles and the per-block arithmetic:
//   prefill_tc_kernel             one CTA per item (launches of at most one
//                                 wave: 2 CTAs per SM); row r = head * TPT +
//                                 token; the softmax threads load the query rows.
//                                 In launches of at most one CTA per SM its
//                                 key blocks are split over two groups of the
//                                 CTA (NG = 2), merged in the epilogue.
//   prefill_tc_lean_kernel        larger launches: 3 persistent CTAs per SM
//                                 claiming items, 128 TMEM columns each, P in
//                                 shared memory (described at the kernel).
//   prefill_tc_persistent_kernel  (PKV_PREFILL_LEAN=0) at most 2 CTAs per SM,
//                                 each walking its share of the items: TMEM and
//                                 barriers are set up once, the producer loads
//                                 each item's query tile by TMA into a double
//                                 buffer (row r = token * G + head) ahead of its
//                                 K/V blocks, and O is double-buffered in TMEM so
//                                 one item's epilogue overlaps the next item's MMAs.
// Warp roles (prefill_tc_kernel with NG = 1 and the two-CTA persistent kernel):
//   warp 0      TMA producer: one 2 KiB box per page per K and V (that head's
//               [16 tok][64] slice), 4 pages = one 64-key block per stage,
//               4 stages; pages past the tile's last visible key read the
//               zero fill of a negative coordinate.
//   warp 1      allocates 256 TMEM columns; one thread issues the MMAs:
//                 S_j  [128 x 64]  = Q [128 x 64] . K_j^T      (SS: A and B
//                                    from shared memory, K-major, 128B swizzle)
//                 O   [128 x 64] += P_j [128 x 64] . V_j        (TS: A = P from
//                                    TMEM, B = V MN-major from shared memory)
//               S is double-buffered in TMEM (columns 0-63 / 64-127), P is
//               written over the first 32 columns of its S buffer as packed
//               16-bit pairs, O lives in columns 128-191 (and 192-255, the
//               persistent kernel's second O buffer). Completion is signalled
//               with tcgen05.commit to mbarriers.
//   warps 2-5   softmax, one thread per row (warp w reads TMEM lanes
//               32*(w%4) .. +31): tcgen05.ld of the row's 64 scores, scale,
//               bottom-right causal mask key <= kv_len - q_len + j (which also
//               masks the unwritten tail of the last page), running max with a
//               lazy O rescale (only when the max grows by more than 2^8),
//               exp2, P to TMEM with tcgen05.st; epilogue O / l -> global.
// The unwritten tail rows of the sequence's last page are zeroed in the V
// stage before its P.V MMA, so stale (even NaN) data there meets P = 0 as 0.
//
// Semantics are PagedTorchBackend.attend's (serving/backends/paged_torch.py:
// 400-485): GQA head h reads KV head h // G, pages in listed order, mask
// triu(diag = kv_len - q_len + 1).
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int TC_D = 64;                      // head_dim
constexpr int TC_P = 16;                      // tokens per page
constexpr int TC_ROWS = 128;                  // query rows per CTA (UMMA M)
constexpr int TC_KB = 64;                     // keys per block (UMMA N of S)
constexpr int TC_PPB = TC_KB / TC_P;          // pages per block
constexpr int TC_NST = 4;                     // K/V stages
constexpr int TC_PAGE = TC_P * TC_D * 2;      // 2 KiB: one head's slice of a page
constexpr int TC_KTILE = TC_KB * TC_D * 2;    // 8 KiB
constexpr int TC_STAGE = 2 * TC_KTILE;        // K + V
constexpr int TC_QTILE = TC_ROWS * TC_D * 2;  // 16 KiB
constexpr int TC_TMEM_COLS = 256;
constexpr int TC_THREADS = 192;
constexpr float TC_RESCALE = 8.f;             // rescale O when the max grows by > 2^8

struct TcArgs {
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
  int n_seqs, n_tokens, n_heads, n_kv, layer;
  float scale_log2;
  int early_ctas;  // CTAs [0, early_ctas) are the first wave: they read the plan before griddepcontrol.wait
  int32_t* claim;  // [2] the lean kernel's next item to claim and CTAs finished (zeroed by the plan kernel)
};

// ---------------------------------------------------------------- tcgen05 helpers
// Shared-memory matrix descriptor, 128B swizzle: start address, leading byte
// offset 16 B (unused by swizzled K-major; one 64-element atom in MN), stride
// byte offset 1024 B between 8-row groups, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulate, A/B element format
// (0 = f16, 1 = bf16, always equal), A K-major, B K- or MN-major, N, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(int fmt, int b_mn_major, int n) {
  return (1u << 4) | (uint32_t(fmt) << 7) | (uint32_t(fmt) << 10) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(TC_ROWS >> 4) << 24);
}
__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued so far completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

#define PKV_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define PKV_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// 32 consecutive 32-bit TMEM columns of this thread's lane; waits for the load
// inside the same asm statement, so the registers are valid when it returns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : PKV_R8(0), PKV_R8(8), PKV_R8(16), PKV_R8(24)
      : "r"(taddr)
      : "memory");
}
// 64 consecutive 32-bit TMEM columns (two loads, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : PKV_R8(0), PKV_R8(8), PKV_R8(16), PKV_R8(24), PKV_R8(32), PKV_R8(40), PKV_R8(48), PKV_R8(56)
      : "r"(taddr), "r"(taddr + 32)
      : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane <- r; waits for the store.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      PKV_W8(0), PKV_W8(8), PKV_W8(16), PKV_W8(24)
      : "memory");
}
#undef PKV_R8
#undef PKV_W8

// Packed fp32 pairs (sm_100's two-wide FMA / add) and a three-input max: the
// softmax threads are bound by instruction issue, so each pair of scores
// takes one FMA and one add instead of two each.
__device__ __forceinline__ unsigned long long f32x2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f32x2_split(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ int tc_tile_pages(int64_t kv, int ql, int j0, int qt) {
  if (kv < ql || ql < 1) return 0;
  const int jl = min(j0 + qt, ql) - 1;
  return int((kv - ql + jl) / TC_P + 1);
}

// One CTA per item. NG = 1: the tile's key blocks in one chain (two CTAs per
// SM). NG = 2 (launches of at most one CTA per SM, where the longest tile's
// chain of blocks is the launch's critical path): the blocks are split
// between two groups of the CTA, even blocks and odd blocks, each with its own
// MMA warp, K/V ring, S buffers and O in TMEM (columns 256 g .. 256 g + 191)
// and softmax warpgroup; group 1 publishes its rows' (max, sum) in shared
// memory and group 0 merges both O accumulators in the epilogue. The two
// chains share the SM's exponential unit, which one chain leaves two thirds
// idle.
template <typename T, int G, int NG>
__global__ void __launch_bounds__(NG == 1 ? TC_THREADS : 384, NG == 1 ? 2 : 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap, const TcArgs a) {
  constexpr int TPT = TC_ROWS / G;  // tokens per tile
  constexpr int SMW = NG == 1 ? 2 : 4;  // first softmax warp
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = smem;                    // [128 rows][128 B], 128B swizzle
  unsigned char* stages = smem + TC_QTILE;     // NG x TC_NST x {K [64][128 B], V [64][128 B]}
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + size_t(NG) * TC_NST * TC_STAGE);
  // per group g: full[TC_NST], empty[TC_NST] (P.V of the stage's block completed),
  // s_full[2] (S block in TMEM), p_full[2] (P in TMEM and O rescaled, 128
  // arrivals), o_done[2] (P.V of local block jp done: o_done[jp & 1]), drain
  constexpr int NBG = 2 * TC_NST + 7;
  auto gbar = [&](int g) { return bars + g * NBG; };
  uint64_t* q_ready = bars + NG * NBG;         // Q tile in shared memory, 128 arrivals
  uint64_t* b_done = q_ready + 1;              // group 1 published (max, sum) and its O is final, 128 arrivals
  float2* s_ml = reinterpret_cast<float2*>(b_done + 1);  // [128] group 1's (max, sum) per row
  __shared__ uint32_t s_tmem;
  __shared__ int s_bad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_idx = int(blockIdx.x) / a.n_kv, h = int(blockIdx.x) % a.n_kv;
  pdl_trigger();
  // A CTA of the first wave may start while the kernel before it (this
  // layer's append, the previous layer's attention) still runs: up to
  // pdl_wait() it reads only the plan's tile list and the step's BatchMeta,
  // both written before the plan kernel completed (that kernel lets nothing
  // start before then and fences its stores), through L2 (ld.global.cg: no line
  // this SM cached earlier), and checks the tile's page ids. Later CTAs find
  // the earlier kernels long finished: they wait first and read through L1,
  // where the CTAs of one sequence share the lines.
  const bool early = int(blockIdx.x) < a.early_ctas;  // uniform over the CTA
  if (!early) pdl_wait();
  auto ld = [&](const int32_t* p) -> int32_t { return early ? __ldcg(p) : *p; };
  if (tile_idx >= ld(a.n_tiles)) return;
  const int2 tile = early ? __ldcg(a.tiles + tile_idx) : a.tiles[tile_idx];
  const int s = tile.x, j0 = tile.y;
  bool bad = s < 0 || s >= a.n_seqs;
  int q0 = 0, ql = 0, lpl = 0;
  int64_t pa = 0, pb = 0;
  if (!bad) {
    q0 = ld(a.cu_q + s);
    ql = ld(a.cu_q + s + 1) - q0;
    pa = ld(a.kv_indptr + s);
    pb = ld(a.kv_indptr + s + 1);
    lpl = ld(a.last_page_len + s);
  }
  const int64_t npages64 = pb - pa;
  const int64_t kv64 = (npages64 - 1) * TC_P + lpl;
  bad = bad || npages64 < 1 || pa < 0 || pb > a.total_pages || lpl < 1 || lpl > TC_P || ql < 1 ||
        j0 < 0 || j0 >= ql || kv64 < ql || kv64 >= 0x7fffffff || q0 < 0 || q0 + ql > a.n_tokens;
  if (!bad && a.kv_lens && ld(a.kv_lens + s) != kv64) bad = true;
  const int kv = bad ? 0 : int(kv64);
  const int npages = bad ? 0 : int(npages64);
  const int n_pg = bad ? 0 : tc_tile_pages(kv, ql, j0, TPT);  // pages with keys visible to the tile
  const int nblk = (n_pg + TC_PPB - 1) / TC_PPB;
  auto check_pages = [&]() {
    if (threadIdx.x == 0) s_bad = bad ? 1 : 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_pg; i += blockDim.x) {
      const int id = ld(a.kv_indices + pa + i);
      if (id < 0 || id >= a.num_blocks) s_bad = 2;
    }
  };
  if (early) {
    check_pages();
    // warm L2 with this head's slices of the tile's first two key blocks: a
    // hint only (the loads after the wait read through L2, where this layer's
    // appended rows land too), so it may run before the wait
    if (warp == 0 && lane < min(n_pg, 2 * TC_PPB)) {
      const int id = __ldcg(a.kv_indices + pa + lane);
      if (id >= 0 && id < a.num_blocks) {
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, h, 2 * a.layer);
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, h, 2 * a.layer + 1);
      }
    }
    pdl_wait();  // q and this layer's appended rows are written by earlier kernels
  }
  // The query rows, loaded by the first softmax warpgroup now so the loads
  // travel while the page ids are checked (later CTAs) and the barriers and
  // tensor memory are set up; they are stored to shared memory (swizzled)
  // further down.
  const int grp = warp >= SMW ? (warp - SMW) >> 2 : -1;  // softmax group of this warp
  const int r_sm = (warp & 3) * 32 + lane;  // a softmax thread's row
  const int jq_sm = j0 + r_sm % TPT;
  uint4 qv[8];
  if (grp == 0) {
    const bool qok = !bad && jq_sm < ql;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) +
                                                       ((int64_t(q0) + (qok ? jq_sm : 0)) * a.n_heads + h * G + r_sm / TPT) * TC_D);
#pragma unroll
    for (int c = 0; c < 8; ++c) qv[c] = qok ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  if (!early) check_pages();
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int g = 0; g < NG; ++g) {
      uint64_t* b = gbar(g);
      for (int i = 0; i < TC_NST; ++i) {
        mbar_init(&b[i], 1);            // full
        mbar_init(&b[TC_NST + i], 1);   // empty
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&b[2 * TC_NST + i], 1);      // s_full
        mbar_init(&b[2 * TC_NST + 2 + i], 128);  // p_full
        mbar_init(&b[2 * TC_NST + 4 + i], 1);  // o_done
      }
      mbar_init(&b[2 * TC_NST + 6], 1);  // drain
    }
    mbar_init(q_ready, 128);
    mbar_init(b_done, 128);
    fence_mbar_init();
  }
  __syncthreads();

  T* out = static_cast<T*>(a.out);
  // row r of the tile: query head h * G + r / TPT, chunk-relative token j0 + r % TPT
  auto out_row = [&](int r) -> T* {
    const int j = j0 + r % TPT;
    return j < ql ? out + ((int64_t(q0) + j) * a.n_heads + h * G + r / TPT) * TC_D : nullptr;
  };
  if (s_bad) {  // before any TMA or TMEM use
    if (threadIdx.x == 0) flag(a.st, s_bad == 1 ? PKV_DEV_META_BAD : PKV_DEV_SLOT_OOB);
    if (s_bad == 2 && grp == 0) {
      if (T* o = out_row(r_sm))
        for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(o)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }

  // ---- tensor memory: 256 columns per group (S0, S1, O), freed on every path below
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(TC_TMEM_COLS * NG)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tmem;
  // local blocks of group g: global blocks g, g + NG, g + 2 NG, ...
  auto nb_of = [&](int g) { return nblk > g ? (nblk - g + NG - 1) / NG : 0; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // lane g < NG loads group g's blocks (global blocks g, g + NG, ...), so a
    // group that falls behind does not hold up the other's copies
    if (lane < NG) {
      const int g = lane;
      uint64_t* b = gbar(g);
      const int kvc = 2 * a.layer;
      int issued = 0;  // local blocks of group g issued
      bool dead = false;
      for (int jj = 0; jj * NG + g < nblk; ++jj) {
        const int j = jj * NG + g, st = jj % TC_NST;
        if (jj >= TC_NST && !mbar_wait_bounded_sleepy(&b[TC_NST + st], ((jj / TC_NST) - 1) & 1, a.st, 64)) {
          dead = true;
          break;
        }
        unsigned char* kd = stages + (size_t(g) * TC_NST + st) * TC_STAGE;
        mbar_arrive_expect_tx(&b[st], TC_STAGE);
#pragma unroll
        for (int u = 0; u < TC_PPB; ++u) {
          const int pg = j * TC_PPB + u;
          // a page past the tile's visible keys reads the zero fill of a negative coordinate
          const int row = pg < n_pg ? a.kv_indices[pa + pg] * TC_P : -TC_P;
          tma_load_4d(kd + u * TC_PAGE, &tmap, &b[st], 0, row, h, kvc);
          tma_load_4d(kd + TC_KTILE + u * TC_PAGE, &tmap, &b[st], 0, row, h, kvc + 1);
        }
        issued = jj + 1;
      }
      // let this group's copies land before the CTA's shared memory can be released
      if (dead)
        for (int i = max(0, issued - TC_NST); i < issued; ++i) mbar_wait_bounded(&b[i % TC_NST], (i / TC_NST) & 1, nullptr);
    }
  } else if (warp >= 1 && warp <= NG) {
    // ------------------------------------------------------------ MMA issuer of group warp - 1
    const int g = warp - 1;
    uint64_t* b = gbar(g);
    uint64_t* full = b;
    uint64_t* empty = b + TC_NST;
    uint64_t* s_full = b + 2 * TC_NST;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_done = s_full + 4;
    uint64_t* drain = s_full + 6;
    const uint32_t tg = tbase + g * TC_TMEM_COLS;
    const uint32_t tO = tg + 128;
    const int nb = nb_of(g);
    constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    constexpr uint32_t idS = idesc_f16(fmt, 0, TC_KB);
    constexpr uint32_t idPV = idesc_f16(fmt, 1, TC_D);
    const uint32_t q_addr = smem_u32(qs);
    unsigned char* gst = stages + size_t(g) * TC_NST * TC_STAGE;
    bool dead = !mbar_wait_bounded(q_ready, 0, a.st);
    dead = __any_sync(0xffffffffu, dead);
    const int lp_blk = (npages - 1) / TC_PPB;  // global block holding the sequence's last page
    for (int j = 0; j <= nb && !dead; ++j) {
      if (j < nb) {
        const int st = j % TC_NST, jg = j * NG + g;
        if (!mbar_wait_bounded(&full[st], (j / TC_NST) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        if (jg == lp_blk && lpl < TC_P && npages - 1 < n_pg) {
          // rows lpl..15 of the last page's V slice were never written: zero them
          uint4* vt = reinterpret_cast<uint4*>(gst + size_t(st) * TC_STAGE + TC_KTILE +
                                               (npages - 1 - jg * TC_PPB) * TC_PAGE);
          for (int r = lpl * 8 + lane; r < TC_P * 8; r += 32) vt[r] = make_uint4(0u, 0u, 0u, 0u);
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) {
          tc_fence_after();
          const uint32_t kaddr = smem_u32(gst + size_t(st) * TC_STAGE);
          const uint32_t dS = tg + (j & 1) * TC_KB;
#pragma unroll
          for (int k = 0; k < TC_D / 16; ++k)
            umma_ss(dS, sw128_desc(q_addr + 32 * k), sw128_desc(kaddr + 32 * k), idS, k > 0);
          umma_commit(&s_full[j & 1]);
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int jp = j - 1, stp = jp % TC_NST;
        if (!mbar_wait_bounded(&p_full[jp & 1], (jp >> 1) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        if (lane == 0) {
          tc_fence_after();
          const uint32_t vaddr = smem_u32(gst + size_t(stp) * TC_STAGE + TC_KTILE);
          const uint32_t aP = tg + (jp & 1) * TC_KB;
#pragma unroll
          for (int k = 0; k < TC_KB / 16; ++k)
            umma_ts(tO, aP + 8 * k, sw128_desc(vaddr + 16 * 128 * k), idPV, (jp > 0 || k > 0) ? 1u : 0u);
          umma_commit(&o_done[jp & 1]);
          umma_commit(&empty[stp]);
        }
        __syncwarp();
      }
    }
    // every MMA issued above has completed before TMEM is freed
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, a.st);
    }
    __syncwarp();
  } else if (grp >= 0) {
    // ------------------------------------------------------------ softmax warps of group grp
    const int g = grp;
    uint64_t* s_full = gbar(g) + 2 * TC_NST;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_done = s_full + 4;
    const uint32_t tg = tbase + g * TC_TMEM_COLS;
    const uint32_t tO = tg + 128;
    const int nb = nb_of(g);
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const int r = r_sm;
    const int jq = jq_sm;
    const bool valid = jq < ql;
    const int lim = valid ? kv - ql + jq : -1;  // last visible key of this row
    if (g == 0) {
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(qs + r * 128 + ((c ^ (r & 7)) << 4)) = qv[c];
      fence_proxy_async_smem();
      mbar_arrive(q_ready);
    }
    const uint32_t lane_off = uint32_t(q4 * 32) << 16;
    const float sl2 = a.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool dead = false;
    // Waits on o_done[x] happen in phase order on each barrier: block j always
    // waits for P.V of block j - 2 (its P buffer is about to be overwritten) and,
    // only when it rescales O, for P.V of block j - 1 — so a try_wait on a
    // parity never meets a barrier two phases ahead.
    for (int j = 0; j < nb; ++j) {
      const int b = j & 1;
      if (!mbar_wait_bounded(&s_full[b], (j >> 1) & 1, a.st)) dead = true;
      if (j >= 2 && !dead && !mbar_wait_bounded(&o_done[b], ((j - 2) >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld64(tg + lane_off + b * TC_KB, sr);
      const int kb0 = (j * NG + g) * TC_KB;
      if (sl2 <= 0.f) {  // a non-positive scale: scale first so the masked -inf stays the minimum
#pragma unroll
        for (int i = 0; i < 64; ++i) sr[i] = __float_as_uint(__uint_as_float(sr[i]) * sl2);
      }
      if (kb0 + TC_KB - 1 > lim) {  // the block reaches past this row's last visible key
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (kb0 + i > lim) sr[i] = __float_as_uint(-INFINITY);
      }
      float mx;
      {
        float t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t[u] = __uint_as_float(sr[u]);
#pragma unroll
        for (int i = 8; i < 64; i += 2)
          t[(i >> 1) & 7] = max3f(t[(i >> 1) & 7], __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
        mx = max3f(max3f(t[0], t[1], t[2]), max3f(t[3], t[4], t[5]), fmaxf(t[6], t[7]));
      }
      const float sc = sl2 > 0.f ? sl2 : 1.f;  // the scale still to apply (log2 units)
      mx = mx * sc;                            // -inf stays -inf (sc > 0)
      const float mn = fmaxf(m, mx);
      float m_new = m;
      if (mn != -INFINITY && (m == -INFINITY || mn > m + TC_RESCALE)) m_new = mn;
      const bool resc = (m_new != m) && (m != -INFINITY);  // earlier blocks already added to O
      const float alpha = resc ? ex2(m - m_new) : 1.f;
      l *= alpha;
      m = m_new;
      if (__any_sync(0xffffffffu, resc)) {
        // O holds P.V up to block j - 1: let that finish before reading it
        if (j >= 1 && !mbar_wait_bounded(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        tc_fence_after();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + hf * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + lane_off + hf * 32, o);
        }
      }
      const float mu = m == -INFINITY ? 0.f : m;
      const unsigned long long sc2 = f32x2(sc, sc), nmu2 = f32x2(-mu, -mu);
      unsigned long long lt2[4] = {0ull, 0ull, 0ull, 0ull};  // pairs of running sums (0.f bits)
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x0, x1;
        f32x2_split(fma_f32x2(f32x2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nmu2), x0, x1);
        const float p0 = ex2(x0), p1 = ex2(x1);
        lt2[i & 3] = add_f32x2(lt2[i & 3], f32x2(p0, p1));
        pk[i] = MmaOp<T>::pack(p0, p1);
      }
      float lt[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) f32x2_split(lt2[u], lt[2 * u], lt[2 * u + 1]);
      const float ls = ((lt[0] + lt[1]) + (lt[2] + lt[3])) + ((lt[4] + lt[5]) + (lt[6] + lt[7]));
      l += ls;
      tmem_st32(tg + lane_off + b * TC_KB, pk);
      tc_fence_before();
      mbar_arrive(&p_full[b]);
    }
    // epilogue: P.V of the group's last block done (the barrier's previous
    // phase was waited at block nb - 1)
    if (nb > 0 && !dead && !mbar_wait_bounded(&o_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1, a.st)) dead = true;
    dead = __any_sync(0xffffffffu, dead);
    if (NG == 2 && g == 1) {
      // publish this row's (max, sum); O (if the group had blocks) is final
      s_ml[r] = make_float2(m, l);
      tc_fence_before();
      mbar_arrive(b_done);
    } else if (!dead && nb > 0) {
      float m1 = -INFINITY, l1 = 0.f;
      int nb1 = 0;
      if (NG == 2) {
        if (!mbar_wait_bounded(b_done, 0, a.st)) dead = true;
        const float2 ml = s_ml[r];
        m1 = ml.x;
        l1 = ml.y;
        nb1 = nb_of(1);
      }
      // merge: both parts to the larger of the two maxima (a part without
      // visible keys in this row has max -inf and weight 0)
      const float mm = fmaxf(m, m1);
      const float w0 = m == -INFINITY ? 0.f : ex2(m - mm);
      const float w1 = (nb1 == 0 || m1 == -INFINITY) ? 0.f : ex2(m1 - mm);
      const float lsum = l * w0 + l1 * w1;
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      const float f0 = w0 * inv, f1 = w1 * inv;
      tc_fence_after();
      T* orow = out_row(r);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + hf * 32, o);
        if (NG == 2 && nb1 > 0) {
          uint32_t o1[32];
          tmem_ld32(tbase + TC_TMEM_COLS + 128 + lane_off + hf * 32, o1);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[i] = __float_as_uint(__uint_as_float(o[i]) * f0 + __uint_as_float(o1[i]) * f1);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f0);
        }
        if (!dead && orow) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 v;
            v.x = MmaOp<T>::pack(__uint_as_float(o[8 * c]), __uint_as_float(o[8 * c + 1]));
            v.y = MmaOp<T>::pack(__uint_as_float(o[8 * c + 2]), __uint_as_float(o[8 * c + 3]));
            v.z = MmaOp<T>::pack(__uint_as_float(o[8 * c + 4]), __uint_as_float(o[8 * c + 5]));
            v.w = MmaOp<T>::pack(__uint_as_float(o[8 * c + 6]), __uint_as_float(o[8 * c + 7]));
            reinterpret_cast<uint4*>(orow)[hf * 4 + c] = v;
          }
        }
      }
    }
  }

  // ---- free tensor memory once every role is done with it
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_TMEM_COLS * NG)
                 : "memory");
  }
}

size_t tc_smem(int ng) {
  return 1024 + TC_QTILE + size_t(ng) * TC_NST * TC_STAGE + 8 * (ng * (2 * TC_NST + 7) + 2) + 128 * 8;
}

// 3-D TMA load (the query tile: dims D, query head, token).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                           int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// One work item: a tile of TPT tokens of sequence s (from j0) for KV head h.
struct TcItem {
  int bad;  // metadata inconsistent: the item is skipped by every role (and flagged)
  int h, s, j0, q0, ql, lpl, kv, npages, n_pg, nblk;
  int64_t pa;
};

// Every role derives the same items in the same order from the plan's tile
// list (sorted by pages read, longest first): item w = tile w / n_kv, KV head
// w % n_kv. `l2`: read through L2 (before griddepcontrol.wait).
template <int TPT>
__device__ __forceinline__ TcItem tc_item(const TcArgs& a, int w, bool l2) {
  auto ld = [&](const int32_t* p) -> int32_t { return l2 ? __ldcg(p) : *p; };
  TcItem it;
  const int tile_idx = w / a.n_kv;
  it.h = w - tile_idx * a.n_kv;
  const int2 tile = l2 ? __ldcg(a.tiles + tile_idx) : a.tiles[tile_idx];
  it.s = tile.x;
  it.j0 = tile.y;
  bool bad = it.s < 0 || it.s >= a.n_seqs;
  int q0 = 0, ql = 0, lpl = 0;
  int64_t pa = 0, pb = 0;
  if (!bad) {
    q0 = ld(a.cu_q + it.s);
    ql = ld(a.cu_q + it.s + 1) - q0;
    pa = ld(a.kv_indptr + it.s);
    pb = ld(a.kv_indptr + it.s + 1);
    lpl = ld(a.last_page_len + it.s);
  }
  const int64_t npages64 = pb - pa;
  const int64_t kv64 = (npages64 - 1) * TC_P + lpl;
  bad = bad || npages64 < 1 || pa < 0 || pb > a.total_pages || lpl < 1 || lpl > TC_P || ql < 1 ||
        it.j0 < 0 || it.j0 >= ql || kv64 < ql || kv64 >= 0x7fffffff || q0 < 0 || q0 + ql > a.n_tokens;
  if (!bad && a.kv_lens && ld(a.kv_lens + it.s) != kv64) bad = true;
  it.bad = bad;
  it.q0 = q0;
  it.ql = ql;
  it.lpl = lpl;
  it.pa = pa;
  it.kv = bad ? 0 : int(kv64);
  it.npages = bad ? 0 : int(npages64);
  it.n_pg = bad ? 0 : tc_tile_pages(it.kv, ql, it.j0, TPT);
  it.nblk = (it.n_pg + TC_PPB - 1) / TC_PPB;
  return it;
}

// The CTA's r-th item: rounds of gridDim.x items, walked forward on even rounds
// and backward on odd ones, so that over the longest-first list every CTA's
// total stays close to the others'.
__device__ __forceinline__ int tc_item_index(int r) {
  const int c = int(blockIdx.x), n = int(gridDim.x);
  return r * n + ((r & 1) ? n - 1 - c : c);
}

template <typename T, int G>
__global__ void __launch_bounds__(TC_THREADS, 2) prefill_tc_persistent_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap qmap,
                                                                   const TcArgs a) {
  constexpr int TPT = TC_ROWS / G;  // tokens per tile
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qbuf = smem;                      // 2 x [128 rows][128 B], 128B swizzle
  unsigned char* stages = smem + 2 * TC_QTILE;     // TC_NST x {K [64][128 B], V [64][128 B]}
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + size_t(TC_NST) * TC_STAGE);
  uint64_t* empty = full + TC_NST;                 // P.V of the stage's block completed
  uint64_t* s_full = empty + TC_NST;               // [2] S block in TMEM
  uint64_t* p_full = s_full + 2;                   // [2] P in TMEM (and O rescaled), 128 arrivals
  uint64_t* o_done = p_full + 2;                   // [2] P.V of global block g done: o_done[g & 1]
  uint64_t* q_full = o_done + 2;                   // [2] query tile landed (TMA)
  uint64_t* q_empty = q_full + 2;                  // [2] the item's S MMAs read their query tile
  uint64_t* o_free = q_empty + 2;                  // [2] epilogue read O buffer, 128 arrivals
  uint64_t* pg_bar = o_free + 2;                   // [2] page-id checks of the item gathered, 128 arrivals
  uint64_t* drain = pg_bar + 2;                    // every MMA of the CTA completed
  __shared__ uint32_t s_tmem;
  __shared__ int s_pg_bad[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  // The plan kernel (tile list) completed before this kernel could start and
  // fenced its stores: the item count may be read before griddepcontrol.wait.
  const int n_items = __ldcg(a.n_tiles) * a.n_kv;
  if (int(blockIdx.x) >= n_items) return;  // no item for this CTA (uniform over the CTA)

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    prefetch_tmap(&qmap);
    for (int i = 0; i < TC_NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&o_free[i], 128);
      mbar_init(&pg_bar[i], 128);
      s_pg_bad[i] = 0;
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane < 2 * TC_PPB) {
    // warm L2 with this head's slices of the first item's first two key blocks:
    // a hint (no shared memory written), so it may run before the wait
    const TcItem f = tc_item<TPT>(a, int(blockIdx.x), true);
    if (!f.bad && lane < f.n_pg) {
      const int id = __ldcg(a.kv_indices + f.pa + lane);
      if (id >= 0 && id < a.num_blocks) {
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, f.h, 2 * a.layer);
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, f.h, 2 * a.layer + 1);
      }
    }
  }
  // ---- tensor memory: 256 columns S0 | S1 | O0 | O1, freed on every path below
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tmem;
  pdl_wait();  // q and this layer's appended K/V rows are written by earlier kernels

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int kvc = 2 * a.layer;
      uint32_t g = 0;  // global key-block counter of this CTA
      int it = 0;      // good items started
      bool dead = false;
      for (int r = 0; !dead; ++r) {
        const int w = tc_item_index(r);
        if (w >= n_items) break;
        const TcItem I = tc_item<TPT>(a, w, false);
        if (I.bad) continue;
        const int qb = it & 1;
        if (it >= 2 && !mbar_wait_bounded_sleepy(&q_empty[qb], ((it - 2) >> 1) & 1, a.st, 64)) {
          dead = true;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qb], TC_QTILE);
        tma_load_3d(qbuf + qb * TC_QTILE, &qmap, &q_full[qb], 0, I.h * G, I.q0 + I.j0);
        ++it;
        for (int j = 0; j < I.nblk; ++j, ++g) {
          const int st = int(g % TC_NST);
          if (g >= TC_NST && !mbar_wait_bounded_sleepy(&empty[st], ((g / TC_NST) - 1) & 1, a.st, 64)) {
            dead = true;
            break;
          }
          unsigned char* kd = stages + size_t(st) * TC_STAGE;
          mbar_arrive_expect_tx(&full[st], TC_STAGE);
#pragma unroll
          for (int u = 0; u < TC_PPB; ++u) {
            const int pg = j * TC_PPB + u;
            // a page past the tile's visible keys reads the zero fill of a negative coordinate
            const int row = pg < I.n_pg ? a.kv_indices[I.pa + pg] * TC_P : -TC_P;
            tma_load_4d(kd + u * TC_PAGE, &tmap, &full[st], 0, row, I.h, kvc);
            tma_load_4d(kd + TC_KTILE + u * TC_PAGE, &tmap, &full[st], 0, row, I.h, kvc + 1);
          }
        }
      }
      if (dead) {
        // let this CTA's own copies land before its shared memory can be released
        for (uint32_t i = g > TC_NST ? g - TC_NST : 0; i < g; ++i)
          mbar_wait_bounded(&full[i % TC_NST], (i / TC_NST) & 1, nullptr);
        for (int i = it > 2 ? it - 2 : 0; i < it; ++i) mbar_wait_bounded(&q_full[i & 1], (i >> 1) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    constexpr uint32_t idS = idesc_f16(fmt, 0, TC_KB);
    constexpr uint32_t idPV = idesc_f16(fmt, 1, TC_D);
    uint32_t g = 0;
    int it = 0;
    bool dead = false;
    for (int r = 0; !dead; ++r) {
      const int w = tc_item_index(r);
      if (w >= n_items) break;
      const TcItem I = tc_item<TPT>(a, w, false);
      if (I.bad) continue;
      const int qb = it & 1;
      const uint32_t tO = tbase + 128 + qb * TC_D;
      if (!mbar_wait_bounded(&q_full[qb], (it >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      const uint32_t q_addr = smem_u32(qbuf + qb * TC_QTILE);
      const int lp_blk = (I.npages - 1) / TC_PPB;  // block holding the sequence's last page
      for (int j = 0; j <= I.nblk; ++j) {
        if (j < I.nblk) {
          const uint32_t gj = g + j;
          const int st = int(gj % TC_NST);
          if (!mbar_wait_bounded(&full[st], (gj / TC_NST) & 1, a.st)) dead = true;
          dead = __any_sync(0xffffffffu, dead);
          if (dead) break;
          if (j == lp_blk && I.lpl < TC_P && I.npages - 1 < I.n_pg) {
            // rows lpl..15 of the last page's V slice were never written: zero them
            uint4* vt = reinterpret_cast<uint4*>(stages + size_t(st) * TC_STAGE + TC_KTILE +
                                                 (I.npages - 1 - j * TC_PPB) * TC_PAGE);
            for (int rr = I.lpl * 8 + lane; rr < TC_P * 8; rr += 32) vt[rr] = make_uint4(0u, 0u, 0u, 0u);
            fence_proxy_async_smem();
            __syncwarp();
          }
          if (lane == 0) {
            tc_fence_after();
            const uint32_t kaddr = smem_u32(stages + size_t(st) * TC_STAGE);
            const uint32_t dS = tbase + (gj & 1) * TC_KB;
#pragma unroll
            for (int k = 0; k < TC_D / 16; ++k)
              umma_ss(dS, sw128_desc(q_addr + 32 * k), sw128_desc(kaddr + 32 * k), idS, k > 0);
            umma_commit(&s_full[gj & 1]);
            if (j == I.nblk - 1) umma_commit(&q_empty[qb]);  // the item's last read of its query tile
          }
          __syncwarp();
        }
        if (j >= 1) {
          const uint32_t gp = g + j - 1;
          const int stp = int(gp % TC_NST);
          if (!mbar_wait_bounded(&p_full[gp & 1], (gp >> 1) & 1, a.st)) dead = true;
          // the item's first P.V overwrites this O buffer: the epilogue two items back read it
          if (!dead && j == 1 && it >= 2 && !mbar_wait_bounded(&o_free[qb], ((it - 2) >> 1) & 1, a.st))
            dead = true;
          dead = __any_sync(0xffffffffu, dead);
          if (dead) break;
          if (lane == 0) {
            tc_fence_after();
            const uint32_t vaddr = smem_u32(stages + size_t(stp) * TC_STAGE + TC_KTILE);
            const uint32_t aP = tbase + (gp & 1) * TC_KB;
#pragma unroll
            for (int k = 0; k < TC_KB / 16; ++k)
              umma_ts(tO, aP + 8 * k, sw128_desc(vaddr + 16 * 128 * k), idPV, (j > 1 || k > 0) ? 1u : 0u);
            umma_commit(&o_done[gp & 1]);
            umma_commit(&empty[stp]);
          }
          __syncwarp();
        }
      }
      g += I.nblk;
      ++it;
    }
    // every MMA issued above has completed before TMEM is freed
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, a.st);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    const int q4 = warp & 3;    // TMEM lane quarter this warp may access
    const int r = q4 * 32 + lane;  // this thread's row: token r / G, query head r % G of the item's group
    const uint32_t lane_off = uint32_t(q4 * 32) << 16;
    const float sl2 = a.scale_log2;
    T* out = static_cast<T*>(a.out);
    uint32_t g = 0;
    int it = 0;
    bool dead = false;
    for (int rr = 0; !dead; ++rr) {
      const int w = tc_item_index(rr);
      if (w >= n_items) break;
      const TcItem I = tc_item<TPT>(a, w, false);
      if (I.bad) {
        if (r == 0) flag(a.st, PKV_DEV_META_BAD);
        continue;
      }
      const int qb = it & 1;
      const uint32_t tO = tbase + 128 + qb * TC_D;
      // page ids of the item, checked while its blocks run (gathered at the epilogue)
      bool pg_bad = false;
      for (int p = r; p < I.n_pg; p += 128) {
        const int id = a.kv_indices[I.pa + p];
        pg_bad |= id < 0 || id >= a.num_blocks;
      }
      const int jq = I.j0 + r / G;
      const bool valid = jq < I.ql;
      const int lim = valid ? I.kv - I.ql + jq : -1;  // last visible key of this row
      float m = -INFINITY, l = 0.f;
      // Waits on o_done[x] happen in phase order on each barrier: block gj waits
      // for P.V of block gj - 2 (its P buffer is about to be overwritten) and,
      // only when it rescales O, for P.V of block gj - 1; the epilogue for the
      // item's last block — so a try_wait on a parity never meets a barrier two
      // phases ahead.
      for (int j = 0; j < I.nblk; ++j) {
        const uint32_t gj = g + j;
        const int b = gj & 1;
        if (!mbar_wait_bounded(&s_full[b], (gj >> 1) & 1, a.st)) dead = true;
        if (j >= 2 && !dead && !mbar_wait_bounded(&o_done[b], ((gj - 2) >> 1) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld64(tbase + lane_off + b * TC_KB, sr);
        const int kb0 = j * TC_KB;
        if (sl2 <= 0.f) {  // a non-positive scale: scale first so the masked -inf stays the minimum
#pragma unroll
          for (int i = 0; i < 64; ++i) sr[i] = __float_as_uint(__uint_as_float(sr[i]) * sl2);
        }
        if (kb0 + TC_KB - 1 > lim) {  // the block reaches past this row's last visible key
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kb0 + i > lim) sr[i] = __float_as_uint(-INFINITY);
        }
        float mx;
        {
          float t[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) t[u] = __uint_as_float(sr[u]);
#pragma unroll
          for (int i = 8; i < 64; i += 2)
            t[(i >> 1) & 7] = max3f(t[(i >> 1) & 7], __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          mx = max3f(max3f(t[0], t[1], t[2]), max3f(t[3], t[4], t[5]), fmaxf(t[6], t[7]));
        }
        const float sc = sl2 > 0.f ? sl2 : 1.f;  // the scale still to apply (log2 units)
        mx = mx * sc;                            // -inf stays -inf (sc > 0)
        const float mn = fmaxf(m, mx);
        float m_new = m;
        if (mn != -INFINITY && (m == -INFINITY || mn > m + TC_RESCALE)) m_new = mn;
        const bool resc = (m_new != m) && (m != -INFINITY);  // earlier blocks already added to O
        const float alpha = resc ? ex2(m - m_new) : 1.f;
        l *= alpha;
        m = m_new;
        if (__any_sync(0xffffffffu, resc)) {
          // O holds P.V up to block gj - 1 (j >= 1 here): let that finish before reading it
          if (!mbar_wait_bounded(&o_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1, a.st)) dead = true;
          dead = __any_sync(0xffffffffu, dead);
          if (dead) break;
          tc_fence_after();
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t o[32];
            tmem_ld32(tO + lane_off + hf * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + lane_off + hf * 32, o);
          }
        }
        const float mu = m == -INFINITY ? 0.f : m;
        const unsigned long long sc2 = f32x2(sc, sc), nmu2 = f32x2(-mu, -mu);
        unsigned long long lt2[4] = {0ull, 0ull, 0ull, 0ull};  // pairs of running sums (0.f bits)
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x0, x1;
          f32x2_split(fma_f32x2(f32x2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nmu2), x0,
                      x1);
          const float p0 = ex2(x0), p1 = ex2(x1);
          lt2[i & 3] = add_f32x2(lt2[i & 3], f32x2(p0, p1));
          pk[i] = MmaOp<T>::pack(p0, p1);
        }
        float lt[8];
#pragma unroll
        for (int u = 0; u < 4; ++u) f32x2_split(lt2[u], lt[2 * u], lt[2 * u + 1]);
        const float ls = ((lt[0] + lt[1]) + (lt[2] + lt[3])) + ((lt[4] + lt[5]) + (lt[6] + lt[7]));
        l += ls;
        tmem_st32(tbase + lane_off + b * TC_KB, pk);
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      if (dead) break;
      // ---- epilogue: O / l of the item -> global memory, while the MMA warp
      // goes on with the next item into the other O buffer
      const uint32_t gl = g + I.nblk - 1;
      if (!mbar_wait_bounded(&o_done[gl & 1], (gl >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      tc_fence_after();
      uint32_t o[2][32];
      tmem_ld32(tO + lane_off, o[0]);
      tmem_ld32(tO + lane_off + 32, o[1]);
      tc_fence_before();
      mbar_arrive(&o_free[qb]);
      if (pg_bad) s_pg_bad[qb] = it + 1;
      mbar_arrive(&pg_bar[qb]);
      if (!mbar_wait_bounded(&pg_bar[qb], (it >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      const bool zero = s_pg_bad[qb] == it + 1;  // a page id outside the pool: the item's rows are zeros
      if (zero && r == 0) flag(a.st, PKV_DEV_SLOT_OOB);
      if (valid) {
        T* orow = out + ((int64_t(I.q0) + jq) * a.n_heads + I.h * G + r % G) * TC_D;
        const float inv = (l > 0.f && !zero) ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int e = c * 8;
          uint4 v;
          v.x = MmaOp<T>::pack(__uint_as_float(o[e >> 5][e & 31]) * inv, __uint_as_float(o[e >> 5][(e & 31) + 1]) * inv);
          v.y = MmaOp<T>::pack(__uint_as_float(o[e >> 5][(e & 31) + 2]) * inv, __uint_as_float(o[e >> 5][(e & 31) + 3]) * inv);
          v.z = MmaOp<T>::pack(__uint_as_float(o[e >> 5][(e & 31) + 4]) * inv, __uint_as_float(o[e >> 5][(e & 31) + 5]) * inv);
          v.w = MmaOp<T>::pack(__uint_as_float(o[e >> 5][(e & 31) + 6]) * inv, __uint_as_float(o[e >> 5][(e & 31) + 7]) * inv);
          if (zero) v = make_uint4(0u, 0u, 0u, 0u);
          reinterpret_cast<uint4*>(orow)[c] = v;
        }
      }
      g += I.nblk;
      ++it;
    }
  }

  // ---- free tensor memory once every role is done with it
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_TMEM_COLS)
                 : "memory");
  }
}

size_t tcp_smem() { return 1024 + 2 * size_t(TC_QTILE) + size_t(TC_NST) * TC_STAGE + 256; }

// ------------------------------------------------------------------ lean kernel
// prefill_tc_lean_kernel: the persistent kernel's item walk with three CTAs
// per SM instead of two, so that each SM sub-partition interleaves three
// softmax warps' block chains instead of two. What buys the residency: 128
// TMEM columns per CTA (one S block and one O) and P in shared memory instead
// of tensor memory. With P out of the S columns, the next block's S MMA may
// overwrite S as soon as the softmax threads have loaded it into registers:
// S_{j+1} is computed while the softmax of block j runs, as with two S
// buffers. Shared memory (67 KiB): the query tile, K and V rings of two
// 64-key slots each, and the P tile ([128 rows][64 keys], 128B swizzle, the
// A operand of the P.V MMA). K and V have rings of their own because a K slot
// is free once its block's S MMA completed, a softmax period before the
// block's P.V frees the V slot: the producer loads K two blocks ahead of the
// S MMA that needs it, and the page ids of a block are read before its slots
// are waited for.
// Per block j the softmax threads wait for S_j, load it, release it, find
// the row maximum, wait for P.V_{j-1} (the P tile is free again and O holds
// every earlier block), write P_j and rescale O if needed; the MMA warp
// issues S_{j+1} once S_j is released and K_{j+1} landed, and P.V_j once P_j
// and V_j landed.
constexpr int TL_MINB = 3;          // CTAs per SM
constexpr int TL_NST = 2;           // slots of the K ring and of the V ring
constexpr int TL_TMEM_COLS = 128;   // S in columns 0-63, O in 64-127

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// O row *= alpha (the lazy rescale; rare): out of line, so that the registers
// it needs are saved on its own path and not reserved in the block loop.
__device__ __noinline__ void tl_rescale_o(uint32_t tO, float alpha) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t o[16];
    tmem_ld16(tO + q * 16, o);
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st16(tO + q * 16, o);
  }
}

// exp2(s * sc - mu) of a row's 64 scores, packed to pairs of the pool dtype
// and stored as the row of P in shared memory (16-byte chunk c of row r at
// r * 128 + ((c ^ (r & 7)) << 4): the 128B swizzle of a K-major operand); the
// sum of the exponentials is added to `l`.
template <typename T>
__device__ __forceinline__ void tl_exp64_smem(const uint32_t (&s)[64], unsigned long long sc2,
                                              unsigned long long nmu2, float& l, unsigned char* prow, int r) {
  unsigned long long lt2[2] = {0ull, 0ull};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = c * 8 + 2 * i;
      float x0, x1;
      f32x2_split(fma_f32x2(f32x2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), sc2, nmu2), x0, x1);
      const float p0 = ex2(x0), p1 = ex2(x1);
      lt2[i & 1] = add_f32x2(lt2[i & 1], f32x2(p0, p1));
      pk[i] = MmaOp<T>::pack(p0, p1);
    }
    *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  float a0, a1, b0, b1;
  f32x2_split(lt2[0], a0, a1);
  f32x2_split(lt2[1], b0, b1);
  l += (a0 + a1) + (b0 + b1);
}

// A CTA of the lean kernel is done with the claim counter: the last one of
// the launch zeroes both counters for the next launch with the same plan
// (which claims only after its griddepcontrol.wait, i.e. after this launch
// completed).
__device__ __forceinline__ void tl_count_exit(int32_t* claim) {
  __threadfence();
  if (atomicAdd(claim + 1, 1) == int(gridDim.x) - 1) {
    claim[0] = 0;
    claim[1] = 0;
    __threadfence();
  }
}

// An item's fields as the lean kernel's producer publishes them (nblk = 0:
// no more items; zero: a page id outside the pool, the item's rows are zeros).
struct TlItem {
  int h, q0, j0, ql, kv, npages, lpl, n_pg, nblk, zero;
};

template <typename T, int G>
// 96 registers a thread: three CTAs put up to five warps of 32 x 96 registers
// on an SM sub-partition (16K registers each); 112 would fit only four
__global__ void __launch_bounds__(TC_THREADS, TL_MINB) prefill_tc_lean_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap qmap, const TcArgs a) {
  constexpr int TPT = TC_ROWS / G;  // tokens per tile
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qbuf = smem;                             // [128 rows][128 B], 128B swizzle
  unsigned char* kst = smem + TC_QTILE;                   // TL_NST x K [64 keys][128 B]
  unsigned char* vst = kst + size_t(TL_NST) * TC_KTILE;   // TL_NST x V [64 keys][128 B]
  unsigned char* pbuf = vst + size_t(TL_NST) * TC_KTILE;  // P [128 rows][128 B], 128B swizzle
  uint64_t* kfull = reinterpret_cast<uint64_t*>(pbuf + TC_QTILE);
  uint64_t* kempty = kfull + TL_NST;  // S of the slot's block completed
  uint64_t* vfull = kempty + TL_NST;
  uint64_t* vempty = vfull + TL_NST;  // P.V of the slot's block completed
  uint64_t* s_full = vempty + TL_NST; // S block in TMEM
  uint64_t* s_free = s_full + 1;      // S loaded by the softmax threads, 128 arrivals
  uint64_t* p_full = s_free + 1;      // P in shared memory (and O rescaled), 128 arrivals
  uint64_t* pv_done = p_full + 1;     // P.V of the block completed (P tile free, O updated)
  uint64_t* q_full = pv_done + 1;     // query tile landed (TMA)
  uint64_t* q_empty = q_full + 1;     // the item's S MMAs read the query tile
  uint64_t* o_free = q_empty + 1;     // epilogue read O, 128 arrivals
  uint64_t* item_full = o_free + 1;   // [2] the producer published the item's fields
  uint64_t* item_empty = item_full + 2;  // [2] the MMA warp and the softmax threads are done with them, 129 arrivals
  uint64_t* drain = item_empty + 2;   // every MMA of the CTA completed
  __shared__ uint32_t s_tmem;
  __shared__ TlItem s_item[2];        // the items, in the order every role walks them

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  // The plan kernel (tile list) completed before this kernel could start and
  // fenced its stores: the item count may be read before griddepcontrol.wait.
  const int n_items = __ldcg(a.n_tiles) * a.n_kv;
  if (int(blockIdx.x) >= n_items) {  // no item for this CTA (uniform over the CTA)
    pdl_wait();                      // the counters belong to the previous launch until it completed
    if (threadIdx.x == 0) tl_count_exit(a.claim);
    return;
  }

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    prefetch_tmap(&qmap);
    for (int i = 0; i < TL_NST; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_free, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 129);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane < 2 * TC_PPB) {
    // warm L2 with this head's slices of the first item's first two key blocks:
    // a hint (no shared memory written), so it may run before the wait
    const TcItem f = tc_item<TPT>(a, int(blockIdx.x), true);
    if (!f.bad && lane < f.n_pg) {
      const int id = __ldcg(a.kv_indices + f.pa + lane);
      if (id >= 0 && id < a.num_blocks) {
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, f.h, 2 * a.layer);
        tma_prefetch_l2_4d(&tmap, 0, id * TC_P, f.h, 2 * a.layer + 1);
      }
    }
  }
  // ---- tensor memory: 128 columns S | O, freed on every path below
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(TL_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tmem;
  const uint32_t tO = tbase + TC_KB;
  pdl_wait();  // q and this layer's appended K/V rows are written by earlier kernels

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // Walks the items, checks each one's page ids (all lanes) and publishes its
    // fields in the two-slot item ring, then (lane 0) loads its query tile and
    // its K/V blocks.
    const int kvc = 2 * a.layer;
    uint32_t kiss = 0, viss = 0;  // K / V slots filled so far (global key-block counters)
    int it = 0;                   // items published
    bool dead = false;
    while (!dead) {
      // items are claimed from the front of the longest-first list as CTAs
      // become free (the counter was zeroed by the plan kernel or by the last
      // CTA of the previous launch, which completed before griddepcontrol.wait)
      int w = 0;
      if (lane == 0) w = atomicAdd(a.claim, 1);
      w = __shfl_sync(0xffffffffu, w, 0);
      const bool end = w >= n_items;
      TcItem I{};
      if (!end) {
        I = tc_item<TPT>(a, w, false);
        if (I.bad) {
          if (lane == 0) flag(a.st, PKV_DEV_META_BAD);
          continue;
        }
      }
      bool pg_bad = false;
      for (int pg = lane; pg < I.n_pg; pg += 32) {
        const int id = a.kv_indices[I.pa + pg];
        pg_bad |= id < 0 || id >= a.num_blocks;
      }
      pg_bad = __any_sync(0xffffffffu, pg_bad);
      const int sl = it & 1;
      // the slot is free once every consumer is done with the item two back
      if (it >= 2 && !mbar_wait_bounded_sleepy(&item_empty[sl], ((it - 2) >> 1) & 1, a.st, 32)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      if (lane == 0) {
        TlItem& o = s_item[sl];
        o.h = I.h;
        o.q0 = I.q0;
        o.j0 = I.j0;
        o.ql = I.ql;
        o.kv = I.kv;
        o.npages = I.npages;
        o.lpl = I.lpl;
        o.n_pg = I.n_pg;
        o.nblk = end ? 0 : I.nblk;  // 0: no more items
        o.zero = pg_bad ? 1 : 0;
        if (pg_bad) flag(a.st, PKV_DEV_SLOT_OOB);
        mbar_arrive(&item_full[sl]);
      }
      __syncwarp();
      if (end) break;
      if (lane == 0) {
        if (it >= 1 && !mbar_wait_bounded_sleepy(q_empty, (it - 1) & 1, a.st, 64)) dead = true;
        if (!dead) {
          mbar_arrive_expect_tx(q_full, TC_QTILE);
          tma_load_3d(qbuf, &qmap, q_full, 0, I.h * G, I.q0 + I.j0);
        }
        for (int j = 0; j < I.nblk && !dead; ++j) {
          int rows[TC_PPB];
#pragma unroll
          for (int u = 0; u < TC_PPB; ++u) {
            const int pg = j * TC_PPB + u;
            // a page past the tile's visible keys reads the zero fill of a negative coordinate
            rows[u] = pg < I.n_pg ? a.kv_indices[I.pa + pg] * TC_P : -TC_P;
          }
          const int st = int(kiss % TL_NST);
          if (kiss >= TL_NST && !mbar_wait_bounded_sleepy(&kempty[st], ((kiss / TL_NST) - 1) & 1, a.st, 32)) {
            dead = true;
            break;
          }
          mbar_arrive_expect_tx(&kfull[st], TC_KTILE);
#pragma unroll
          for (int u = 0; u < TC_PPB; ++u)
            tma_load_4d(kst + size_t(st) * TC_KTILE + u * TC_PAGE, &tmap, &kfull[st], 0, rows[u], I.h, kvc);
          ++kiss;
          if (viss >= TL_NST && !mbar_wait_bounded_sleepy(&vempty[st], ((viss / TL_NST) - 1) & 1, a.st, 32)) {
            dead = true;
            break;
          }
          mbar_arrive_expect_tx(&vfull[st], TC_KTILE);
#pragma unroll
          for (int u = 0; u < TC_PPB; ++u)
            tma_load_4d(vst + size_t(st) * TC_KTILE + u * TC_PAGE, &tmap, &vfull[st], 0, rows[u], I.h, kvc + 1);
          ++viss;
        }
      }
      dead = __shfl_sync(0xffffffffu, dead, 0);
      ++it;
    }
    if (dead && lane == 0) {
      // let this CTA's own copies land before its shared memory can be released
      for (uint32_t i = kiss > TL_NST ? kiss - TL_NST : 0; i < kiss; ++i)
        mbar_wait_bounded(&kfull[i % TL_NST], (i / TL_NST) & 1, nullptr);
      for (uint32_t i = viss > TL_NST ? viss - TL_NST : 0; i < viss; ++i)
        mbar_wait_bounded(&vfull[i % TL_NST], (i / TL_NST) & 1, nullptr);
      if (it >= 1) mbar_wait_bounded(q_full, (it - 1) & 1, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    constexpr uint32_t idS = idesc_f16(fmt, 0, TC_KB);
    constexpr uint32_t idPV = idesc_f16(fmt, 1, TC_D);
    const uint32_t q_addr = smem_u32(qbuf), p_addr = smem_u32(pbuf);
    uint32_t g = 0;
    int it = 0;
    bool dead = false;
    // P.V of global block gp (the item's block jp), after its P and its V
    // slot landed; the item's first P.V overwrites O, which the previous
    // item's epilogue reads
    auto pv = [&](uint32_t gp, int jp, const TlItem& I) -> bool {
      const int stp = int(gp % TL_NST);
      bool bad = !mbar_wait_bounded(p_full, gp & 1, a.st);
      if (!bad && jp == 0 && it >= 1 && !mbar_wait_bounded(o_free, (it - 1) & 1, a.st)) bad = true;
      if (!bad && !mbar_wait_bounded(&vfull[stp], (gp / TL_NST) & 1, a.st)) bad = true;
      bad = __any_sync(0xffffffffu, bad);
      if (bad) return false;
      if (jp == (I.npages - 1) / TC_PPB && I.lpl < TC_P && I.npages - 1 < I.n_pg) {
        // rows lpl..15 of the last page's V slice were never written: zero them
        uint4* vt = reinterpret_cast<uint4*>(vst + size_t(stp) * TC_KTILE + (I.npages - 1 - jp * TC_PPB) * TC_PAGE);
        for (int rr = I.lpl * 8 + lane; rr < TC_P * 8; rr += 32) vt[rr] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        tc_fence_after();
        const uint32_t vaddr = smem_u32(vst + size_t(stp) * TC_KTILE);
#pragma unroll
        for (int kk = 0; kk < TC_KB / 16; ++kk)
          umma_ss(tO, sw128_desc(p_addr + 32 * kk), sw128_desc(vaddr + 16 * 128 * kk), idPV,
                  (jp > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&vempty[stp]);
        umma_commit(pv_done);
      }
      __syncwarp();
      return true;
    };
    while (!dead) {
      const int sl = it & 1;
      if (!mbar_wait_bounded(&item_full[sl], (it >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      const TlItem I = s_item[sl];
      if (I.nblk == 0) break;
      if (!mbar_wait_bounded(q_full, it & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      for (int j = 0; j < I.nblk; ++j) {
        const uint32_t gj = g + j;
        const int st = int(gj % TL_NST);
        // S_j overwrites S_{j-1}: after the softmax threads loaded it
        if (gj >= 1 && !mbar_wait_bounded(s_free, (gj - 1) & 1, a.st)) dead = true;
        if (!dead && !mbar_wait_bounded(&kfull[st], (gj / TL_NST) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        if (lane == 0) {
          tc_fence_after();
          const uint32_t kaddr = smem_u32(kst + size_t(st) * TC_KTILE);
#pragma unroll
          for (int kk = 0; kk < TC_D / 16; ++kk)
            umma_ss(tbase, sw128_desc(q_addr + 32 * kk), sw128_desc(kaddr + 32 * kk), idS, kk > 0);
          umma_commit(s_full);
          umma_commit(&kempty[st]);
          if (j == I.nblk - 1) umma_commit(q_empty);  // the item's last read of its query tile
        }
        __syncwarp();
        if (j >= 1 && !pv(gj - 1, j - 1, I)) {
          dead = true;
          break;
        }
      }
      if (dead) break;
      if (!pv(g + I.nblk - 1, I.nblk - 1, I)) {
        dead = true;
        break;
      }
      if (lane == 0) mbar_arrive(&item_empty[sl]);
      g += I.nblk;
      ++it;
    }
    // every MMA issued above has completed before TMEM is freed
    if (lane == 0) {
      umma_commit(drain);
      mbar_wait_bounded(drain, 0, a.st);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    const int q4 = warp & 3;       // TMEM lane quarter this warp may access
    const int r = q4 * 32 + lane;  // this thread's row: token r / G, query head r % G of the item's group
    const uint32_t lane_off = uint32_t(q4 * 32) << 16;
    const float sl2 = a.scale_log2;
    const float sc = sl2 > 0.f ? sl2 : 1.f;  // the scale still to apply after masking (log2 units)
    unsigned char* prow = pbuf + r * 128;
    T* out = static_cast<T*>(a.out);
    uint32_t g = 0;
    int it = 0;
    bool dead = false;
    while (!dead) {
      const int sl = it & 1;
      if (!mbar_wait_bounded(&item_full[sl], (it >> 1) & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      const TlItem I = s_item[sl];
      if (I.nblk == 0) break;
      const int jw0 = I.j0, qlw = I.ql, q0w = I.q0, hw = I.h;  // for the epilogue's stores
      const int jq = I.j0 + r / G;
      const bool valid = jq < I.ql;
      const int lim = valid ? I.kv - I.ql + jq : -1;  // last visible key of this row
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < I.nblk; ++j) {
        const uint32_t gj = g + j;
        if (!mbar_wait_bounded(s_full, gj & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld64(tbase + lane_off, sr);
        tc_fence_before();
        mbar_arrive(s_free);  // S_{j+1} may overwrite S now
        const int kb0 = j * TC_KB;
        if (sl2 <= 0.f) {  // a non-positive scale: scale first so the masked -inf stays the minimum
#pragma unroll
          for (int i = 0; i < 64; ++i) sr[i] = __float_as_uint(__uint_as_float(sr[i]) * sl2);
        }
        if (kb0 + TC_KB - 1 > lim) {  // the block reaches past this row's last visible key
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kb0 + i > lim) sr[i] = __float_as_uint(-INFINITY);
        }
        float mx;
        {
          float t[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) t[u] = __uint_as_float(sr[u]);
#pragma unroll
          for (int i = 8; i < 64; i += 2)
            t[(i >> 1) & 7] = max3f(t[(i >> 1) & 7], __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          mx = max3f(max3f(t[0], t[1], t[2]), max3f(t[3], t[4], t[5]), fmaxf(t[6], t[7]));
        }
        mx = mx * sc;  // -inf stays -inf (sc > 0)
        const float mn = fmaxf(m, mx);
        float m_new = m;
        if (mn != -INFINITY && (m == -INFINITY || mn > m + TC_RESCALE)) m_new = mn;
        const bool resc = (m_new != m) && (m != -INFINITY);  // earlier blocks already added to O
        const float alpha = resc ? ex2(m - m_new) : 1.f;
        l *= alpha;
        m = m_new;
        // P.V_{j-1} done: the P tile is free and O holds every earlier block
        if (gj >= 1 && !mbar_wait_bounded(pv_done, (gj - 1) & 1, a.st)) dead = true;
        dead = __any_sync(0xffffffffu, dead);
        if (dead) break;
        const float mu = m == -INFINITY ? 0.f : m;
        tl_exp64_smem<T>(sr, f32x2(sc, sc), f32x2(-mu, -mu), l, prow, r);
        fence_proxy_async_smem();  // P (generic-proxy stores) -> the P.V MMA (async proxy)
        if (__any_sync(0xffffffffu, resc)) {
          tc_fence_after();
          tl_rescale_o(tO + lane_off, alpha);
        }
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (dead) break;
      // ---- epilogue: O / l of the item -> global memory, then O is released
      // to the next item's first P.V. The rows are staged in this warp's own
      // rows of the P tile (P.V of the item's last block completed, and no
      // other warp writes them), then stored as runs of four whole rows
      // (512 bytes for G = 4: one token's query heads of this KV head).
      const uint32_t gl = g + I.nblk - 1;
      if (!mbar_wait_bounded(pv_done, gl & 1, a.st)) dead = true;
      dead = __any_sync(0xffffffffu, dead);
      if (dead) break;
      tc_fence_after();
      {
        uint32_t o[64];
        tmem_ld64(tO + lane_off, o);
        tc_fence_before();
        mbar_arrive(o_free);  // O read: the next item's first P.V may overwrite it
        const float inv = (l > 0.f && !I.zero) ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int e = c * 8;
          uint4 v;
          v.x = MmaOp<T>::pack(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
          v.y = MmaOp<T>::pack(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
          v.z = MmaOp<T>::pack(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
          v.w = MmaOp<T>::pack(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
          if (I.zero) v = make_uint4(0u, 0u, 0u, 0u);  // a page id outside the pool: the item's rows are zeros
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = v;
        }
      }
      mbar_arrive(&item_empty[sl]);  // this thread has read every field of the item it uses below
      __syncwarp();
      uint4 v[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int rw = q4 * 32 + 4 * kk + (lane >> 3);  // tile row; chunk lane % 8 of it
        v[kk] = *reinterpret_cast<const uint4*>(pbuf + rw * 128 + (((lane & 7) ^ (rw & 7)) << 4));
      }
      __syncwarp();  // the staged rows are read: this warp's next P rows may follow
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int rw = q4 * 32 + 4 * kk + (lane >> 3);
        const int tok = jw0 + rw / G;
        if (tok < qlw)
          reinterpret_cast<uint4*>(out + ((int64_t(q0w) + tok) * a.n_heads + hw * G + rw % G) * TC_D)[lane & 7] = v[kk];
      }
      g += I.nblk;
      ++it;
    }
  }

  // ---- free tensor memory once every role is done with it
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TL_TMEM_COLS)
                 : "memory");
  }
  if (threadIdx.x == 0) tl_count_exit(a.claim);
}

size_t tl_smem() { return 1024 + 2 * size_t(TC_QTILE) + size_t(2 * TL_NST) * TC_KTILE + 256; }

// Which launches the persistent kernel takes: PKV_PREFILL_PERSISTENT unset or 1
// = launches of more than one wave of CTAs, 0 = none (one CTA per tile for every
// launch), 2 = every launch (for tests of the persistent kernel on small batches).
int prefill_persistent_mode() {
  static const int mode = [] {
    const char* e = getenv("PKV_PREFILL_PERSISTENT");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '2') return 2;
    return 1;
  }();
  return mode;
}

// Which persistent kernel runs: PKV_PREFILL_LEAN unset or 1 = the lean kernel
// (three CTAs per SM) for launches of more than one wave, 0 = the two-CTA
// persistent kernel, 2 = the lean kernel for every launch (tests).
int prefill_lean_mode() {
  static const int mode = [] {
    const char* e = getenv("PKV_PREFILL_LEAN");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '2') return 2;
    return 1;
  }();
  return mode;
}

// Whether one-CTA-per-tile launches split each tile's key blocks over two
// groups of the CTA: PKV_PREFILL_SPLIT unset or 1 = launches of at most one CTA
// per SM, 0 = never, 2 = every such launch (tests).
int prefill_split_mode() {
  static const int mode = [] {
    const char* e = getenv("PKV_PREFILL_SPLIT");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '2') return 2;
    return 1;
  }();
  return mode;
}

// Tensor map of the step's query rows q [n_tokens][n_heads][64] as dims
// (D, query head, token): one box = the G heads of one KV head for TPT tokens,
// landing in shared memory as row = token * G + head, 128B-swizzled (the
// layout the S MMA's A operand descriptor reads).
int q_tmap(int32_t dtype, const void* q, int n_tokens, int n_heads, int groups, CUtensorMap* out) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult qr;
    void* fn = nullptr;
    PKV_CUDA_RET(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr));
    if (qr != cudaDriverEntryPointSuccess || !fn)
      return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[3] = {cuuint64_t(TC_D), cuuint64_t(n_heads), cuuint64_t(std::max(n_tokens, 1))};
  const cuuint64_t strides[2] = {cuuint64_t(TC_D) * 2, cuuint64_t(n_heads) * TC_D * 2};
  const cuuint32_t box[3] = {cuuint32_t(TC_D), cuuint32_t(groups), cuuint32_t(TC_ROWS / groups)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt =
      dtype == PKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode(out, dt, 3, const_cast<void*>(q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_CUDA, "cuTensorMapEncodeTiled (q) failed: " + std::to_string(int(r)));
  return PKV_OK;
}


// Launches one of the kernels: `qm` == nullptr -> one CTA per (tile, KV
// head) (prefill_tc_kernel, its key blocks split over `ng` groups), otherwise a
// persistent kernel over `grid` CTAs: prefill_tc_lean_kernel when `lean`, else
// prefill_tc_persistent_kernel.
template <typename T, int G>
int launch_tc_t(const pkv_pool& p, const CUtensorMap& tm, const CUtensorMap* qm, bool lean, int ng,
                const TcArgs& a, int grid, cudaStream_t s) {
  static std::mutex mu;
  static std::vector<char> ready;
  int dev = 0;
  PKV_CUDA_RET(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lock(mu);
    if ((int)ready.size() <= dev) ready.resize(dev + 1, 0);
    if (!ready[dev]) {
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_tc_kernel<T, G, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(tc_smem(1))));
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_tc_kernel<T, G, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(tc_smem(2))));
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_tc_persistent_kernel<T, G>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, int(tcp_smem())));
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_tc_lean_kernel<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(tl_smem())));
      // three CTAs of ~67 KiB need the whole shared-memory carveout
      PKV_CUDA_RET(cudaFuncSetAttribute(prefill_tc_lean_kernel<T, G>,
                                        cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared)));
      ready[dev] = 1;
    }
  }
  if (qm && lean)
    PKV_CUDA_RET(launch_kernel(prefill_tc_lean_kernel<T, G>, dim3(grid), dim3(TC_THREADS), tl_smem(), s, true, tm,
                               *qm, a));
  else if (qm)
    PKV_CUDA_RET(launch_kernel(prefill_tc_persistent_kernel<T, G>, dim3(grid), dim3(TC_THREADS), tcp_smem(), s,
                               true, tm, *qm, a));
  else if (ng == 2)
    PKV_CUDA_RET(launch_kernel(prefill_tc_kernel<T, G, 2>, dim3(grid), dim3(384), tc_smem(2), s, true, tm, a));
  else
    PKV_CUDA_RET(launch_kernel(prefill_tc_kernel<T, G, 1>, dim3(grid), dim3(TC_THREADS), tc_smem(1), s, true, tm, a));
  return PKV_OK;
}

template <typename T>
int launch_tc_g(const pkv_pool& p, int groups, const CUtensorMap& tm, const CUtensorMap* qm, bool lean, int ng,
                const TcArgs& a, int grid, cudaStream_t s) {
  switch (groups) {
    case 1: return launch_tc_t<T, 1>(p, tm, qm, lean, ng, a, grid, s);
    case 2: return launch_tc_t<T, 2>(p, tm, qm, lean, ng, a, grid, s);
    case 4: return launch_tc_t<T, 4>(p, tm, qm, lean, ng, a, grid, s);
    case 8: return launch_tc_t<T, 8>(p, tm, qm, lean, ng, a, grid, s);
  }
  return fail(PKV_ERR_UNSUPPORTED, "tcgen05 prefill kernel: unsupported GQA group size");
}

}  // namespace

int prefill_tc_tile_tokens(int n_heads, int n_kv_heads) { return TC_ROWS / (n_heads / n_kv_heads); }

int prefill_tc_attend(const pkv_pool& p, int layer, int n_heads, const void* q, void* out, float scale,
                      const pkv_batch& b, const int2* tiles, const int32_t* n_tiles, int64_t tiles_cap,
                      cudaStream_t s) {
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(PKV_ERR_ARG, "q and out must be 16-byte aligned");
  CUtensorMap tm;
  if (int rc = pool_tmap_head(p, &tm)) return rc;
  TcArgs a;
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
  a.n_kv = p.n_kv_heads;
  a.layer = layer;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.early_ctas = 2 * num_sms();  // two CTAs per SM (__launch_bounds__ and shared memory)
  a.claim = const_cast<int32_t*>(n_tiles) + 1;  // the plan's workspace: n_tiles[1..2]
  const int qt = prefill_tc_tile_tokens(n_heads, p.n_kv_heads);
  const int64_t bound = std::min<int64_t>((int64_t(b.n_tokens) + qt - 1) / qt + b.n_seqs, tiles_cap);
  const int64_t items = std::max<int64_t>(1, bound) * p.n_kv_heads;
  const int groups = n_heads / p.n_kv_heads;
  const int64_t slots = int64_t(2) * num_sms();  // resident CTAs (two per SM)
  CUtensorMap qm;
  const CUtensorMap* qmp = nullptr;
  int64_t grid = items;
  const int mode = prefill_persistent_mode(), lean_mode = prefill_lean_mode();
  const bool lean = lean_mode == 2 || (lean_mode == 1 && mode == 1 && items > slots);
  if ((mode == 1 && items > slots) || mode == 2 || lean) {
    // more tiles than one wave: persistent CTAs walk the tiles (each CTA's
    // setup, query loads and epilogues overlap its other tiles' work)
    if (int rc = q_tmap(p.dtype, q, b.n_tokens, n_heads, groups, &qm)) return rc;
    qmp = &qm;
    grid = std::min(items, lean ? int64_t(TL_MINB) * num_sms() : slots);
  }
  if (grid > 0x7fffffff) return fail(PKV_ERR_ARG, "prefill batch too large for one launch");
  // one CTA per tile: a launch of at most one CTA per SM splits each tile's key
  // blocks over two groups of its CTA (the longest tile's chain is the launch)
  const int split_mode = prefill_split_mode();
  const int ng = !qmp && (split_mode == 2 || (split_mode == 1 && items <= num_sms())) ? 2 : 1;
  if (ng == 2) a.early_ctas = num_sms();  // one CTA per SM
  if (p.dtype == PKV_F16) return launch_tc_g<__half>(p, groups, tm, qmp, lean, ng, a, int(grid), s);
  return launch_tc_g<__nv_bfloat16>(p, groups, tm, qmp, lean, ng, a, int(grid), s);
}

}  // namespace pkv
