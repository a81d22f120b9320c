/*
 * pkv.h — C ABI of the B200 paged-KV hot path (libpkv.so).
 *
 * Plain pointers, sizes and a CUDA stream handle; no torch or C++ types.
 * Every function returns an int status (PKV_OK on success) and never aborts;
 * pkv_last_error() returns a message for the calling thread's last failure.
 * Arguments are validated on the host before anything touches the device.
 *
 * Device pointers are raw CUDA device addresses; `stream` is a cudaStream_t
 * (NULL = legacy default stream).
 *
 * Pool layout (one allocation per pool, per device):
 *     [num_layers][2 (K,V)][num_blocks][block_size][n_kv_heads][head_dim]
 * so layer l's K (resp. V) is the contiguous slab
 *     base + (2*l + 0|1) * num_blocks * block_size * row_bytes,
 * row_bytes = n_kv_heads * head_dim * elem_size — exactly the per-layer
 * [num_blocks, block_size, n_kv_heads, head_dim] tensors the reference's
 * backends expose as k_pool[l] / v_pool[l] (serving/backends/paged_torch.py:124-137).
 *
 * Page-table inputs follow the reference's BatchMeta contract
 * (docs/ARCHITECTURE.md:88-120): int32 CSR triple kv_indptr / kv_indices /
 * kv_last_page_len, int32 cu_query_lens and slot_mapping.
 */
#ifndef PKV_H_
#define PKV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PKV_API __attribute__((visibility("default")))
#else
#define PKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define PKV_OK 0
#define PKV_ERR_ARG 1          /* invalid argument, detected on the host        */
#define PKV_ERR_UNSUPPORTED 2  /* geometry / dtype no kernel here handles      */
#define PKV_ERR_CUDA 3         /* a CUDA runtime call or launch failed          */
#define PKV_ERR_DEVICE 4       /* a kernel recorded a violation (see flags)     */

/* ---- device status flags (bits of the int32 a kernel may OR into) -------- */
#define PKV_DEV_SLOT_OOB 0x1        /* slot / block id outside the pool          */
#define PKV_DEV_META_BAD 0x2        /* CSR inconsistent (pages vs kv_len, lpl)   */
#define PKV_DEV_QLEN_BAD 0x4        /* decode kernel saw a query length != 1     */
#define PKV_DEV_WAIT_TIMEOUT 0x8    /* a bounded barrier wait gave up            */
#define PKV_DEV_WORKSPACE 0x10      /* workspace smaller than the launch needs   */

/* ---- element types ------------------------------------------------------- */
#define PKV_F16 0
#define PKV_BF16 1
#define PKV_F32 2
#define PKV_F64 3

/* Pool descriptor. All fields are plain values; `base` is a device pointer. */
typedef struct pkv_pool {
  void* base;
  int64_t num_blocks;
  int32_t num_layers;
  int32_t block_size;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t dtype; /* PKV_F16 / PKV_BF16 / PKV_F32 / PKV_F64 */
  int32_t reserved;
} pkv_pool;

/* One step's page table on the device (BatchMeta's fields, int32). */
typedef struct pkv_batch {
  int32_t n_seqs;
  int32_t n_tokens;          /* sum of query lengths (rows of q / out)       */
  int64_t total_pages;       /* kv_indices length == kv_indptr[n_seqs]       */
  const int32_t* cu_query_lens;   /* [n_seqs+1] */
  const int32_t* kv_lens;         /* [n_seqs] (may be NULL: derived from CSR) */
  const int32_t* kv_indptr;       /* [n_seqs+1] */
  const int32_t* kv_indices;      /* [total_pages] */
  const int32_t* kv_last_page_len;/* [n_seqs] */
  int32_t* dev_status;            /* int32 device word kernels OR flags into; may be NULL */
} pkv_batch;

/* ---- library ------------------------------------------------------------- */

/* Library version (major*10000 + minor*100 + patch). */
PKV_API int pkv_version(void);

/* Message of the calling thread's last non-OK status ("" if none). */
PKV_API const char* pkv_last_error(void);

/* ---- KV-append ----------------------------------------------------------
 * Replaces PagedTorchBackend.append_kv (serving/backends/paged_torch.py:209-276)
 * and FlashInferBackend.append_kv (serving/backends/flashinfer_backend.py:443-512):
 * pool.view(-1, H, D)[slot_mapping[t]] = k[t] (and v), for layer `layer`.
 * k, v: device [n_tokens][n_kv_heads][head_dim] contiguous, in the pool dtype.
 * Idempotent. Slots outside [0, num_blocks*block_size) are skipped and flagged
 * PKV_DEV_SLOT_OOB in *dev_status (if given). */
PKV_API int pkv_append_kv(const pkv_pool* pool, int32_t layer, const void* k, const void* v,
                  const int32_t* slot_mapping, int64_t n_tokens, int32_t* dev_status,
                  void* stream);

/* ---- attention ------------------------------------------------------------
 * Replaces PagedTorchBackend.attend (serving/backends/paged_torch.py:280-485) and
 * FlashInferBackend.attend / _ensure_planned (serving/backends/flashinfer_backend.py:516-676):
 * out[t, h] = softmax(scale * q[t,h] . K[s, 0..limit]) V[s, ..] over the
 * sequence's pages in listed order, query head h reading KV head
 * h / (n_heads / n_kv_heads), bottom-right causal limit kv_len - q_len + j.
 * q, out: device [n_tokens][n_heads][head_dim] in the pool dtype.
 *
 * `decode_hint` 1 selects the split-K decode kernel, which requires every
 * query length to be 1 (checked on the device: PKV_DEV_QLEN_BAD). Otherwise a
 * batch with n_tokens != n_seqs (chunked prefill, prefill mixed with decode
 * tokens) runs the tensor-core prefill kernel when the geometry allows (the
 * decode kernel's: fp16/bf16, head_dim 64, 16-token pages, <= 8 KV heads,
 * 1/2/4/8 query heads per KV head), else the generic kernel; with
 * `decode_hint` 0 the batch's q_len == 1 rows run on the decode kernel (a
 * second launch; the plan lists them), with `decode_hint` 2 the caller
 * asserts there are none and that launch is skipped. Workspace
 * (device, 256-byte aligned) of at least pkv_attend_workspace_size() bytes must
 * be given; its counters must be zero before the first call on it and are left
 * zero by every call. */
PKV_API size_t pkv_attend_workspace_size(const pkv_pool* pool, int32_t n_heads, int32_t n_seqs,
                                 int64_t total_pages, int32_t decode_hint);
PKV_API int pkv_attend(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* q, void* out,
               float scale, const pkv_batch* batch, int32_t decode_hint, void* workspace,
               size_t workspace_bytes, void* stream);

/* Build the per-step schedule the attention kernels read (once per step,
 * reused by every layer's pkv_attend_planned with the same batch and
 * workspace): for n_tokens == n_seqs the decode kernel's page descriptors
 * (validating the CSR on the device: PKV_DEV_META_BAD / PKV_DEV_SLOT_OOB /
 * PKV_DEV_QLEN_BAD), otherwise the prefill kernel's tile list, longest tiles
 * first (nothing when only the generic kernel takes the batch). pkv_attend is
 * pkv_plan followed by pkv_attend_planned; a caller attending every layer of
 * one step plans once. The workspace size for a non-decode step is
 * pkv_attend_workspace_size(..., decode_hint = 0). A non-decode plan also
 * lists the batch's q_len == 1 rows for the decode kernel. */
PKV_API int pkv_plan(const pkv_pool* pool, int32_t n_heads, const pkv_batch* batch, void* workspace,
             size_t workspace_bytes, void* stream);
PKV_API int pkv_attend_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* q,
                       void* out, float scale, const pkv_batch* batch, int32_t decode_hint,
                       void* workspace, size_t workspace_bytes, void* stream);

/* KV-append and attention of one layer in one call: pkv_append_kv followed by
 * pkv_attend_planned, with the same arguments and result. For a decode batch
 * (decode_hint 1) on the decode kernel's geometry it is ONE launch: the
 * decode kernel writes each row's new K/V to its slot and patches it into the
 * staged copy of the sequence's last page, which must be the token's slot
 * (the last written position of that page, as in every decode step;
 * PKV_DEV_META_BAD otherwise). Other batches take the two calls. No
 * counterpart in the reference (its engine calls append_kv then attend per
 * layer, docs/ARCHITECTURE.md:167-172). */
PKV_API int pkv_append_attend_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* k,
                              const void* v, const int32_t* slot_mapping, const void* q, void* out,
                              float scale, const pkv_batch* batch, int32_t decode_hint, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Rotary position embedding of q and k at each token's position, the step the
 * engine runs on the projected q and k before append_kv / attend
 * (docs/ARCHITECTURE.md:167-172: project Q/K/V, RoPE at meta.positions,
 * append, attend; the engine itself is not in the reference tree). q [n_tokens]
 * [n_heads][head_dim] and k [n_tokens][n_kv_heads][head_dim] (dtype PKV_F16 or
 * PKV_BF16, contiguous) are rotated into q_out / k_out (which may equal q / k:
 * in place); either tensor may be skipped with 0 heads. Pair (i, i + D/2) of
 * each head of token t is rotated by the angle whose cosine / sine are
 * rope_cos / rope_sin[positions[t]][i] (fp32 tables [rope_max_pos][D/2]):
 * a' = a*cos - b*sin, b' = a*sin + b*cos, every product rounded to fp32 before
 * the difference / sum, then rounded to the dtype (nearest even) — the same
 * bits as that formula evaluated elementwise in fp32. One launch on `stream`.
 * A position outside [0, rope_max_pos) leaves its token unrotated and sets
 * PKV_DEV_META_BAD in *dev_status. */
PKV_API int pkv_rope(int32_t dtype, const void* q, void* q_out, int32_t n_heads, const void* k, void* k_out,
                     int32_t n_kv_heads, int64_t n_tokens, int32_t head_dim, const int64_t* positions,
                     const float* rope_cos, const float* rope_sin, int64_t rope_max_pos, int32_t* dev_status,
                     void* stream);

/* pkv_append_attend_planned with the rotary embedding fused in: q and k are
 * given BEFORE rotation, and the single decode launch rotates each row's q as
 * it loads it and each new K row as it writes it to its slot (tables and
 * rounding as pkv_rope; head_dim 64, so the tables are [rope_max_pos][32],
 * 16-byte aligned). The pool receives the rotated K; q and k are not changed.
 * Same results, bit for bit, as pkv_rope followed by pkv_append_attend_planned.
 * Batches the fused launch does not take (anything but a decode batch on the
 * decode kernel's geometry with 16-byte aligned k and v) return
 * PKV_ERR_UNSUPPORTED with nothing launched: the caller runs those two calls.
 * Replaces the engine's separate RoPE op and append_kv call per layer
 * (docs/ARCHITECTURE.md:167-172); no counterpart in the reference itself. */
PKV_API int pkv_append_attend_rope_planned(const pkv_pool* pool, int32_t layer, int32_t n_heads, const void* k,
                                   const void* v, const int32_t* slot_mapping, const void* q, void* out,
                                   float scale, const pkv_batch* batch, int32_t decode_hint, void* workspace,
                                   size_t workspace_bytes, const int64_t* positions, const float* rope_cos,
                                   const float* rope_sin, int64_t rope_max_pos, void* stream);

/* Which kernel pkv_attend_planned runs for a batch of this shape and hint
 * (host only, nothing touches the device): PKV_KERNEL_GENERIC,
 * PKV_KERNEL_DECODE or PKV_KERNEL_PREFILL; -PKV_ERR_ARG for a bad pool. No
 * counterpart in the reference (its backends have one code path each). */
#define PKV_KERNEL_GENERIC 0
#define PKV_KERNEL_DECODE 1
#define PKV_KERNEL_PREFILL 2
PKV_API int pkv_attend_kernel(const pkv_pool* pool, int32_t n_heads, int32_t n_seqs, int32_t n_tokens,
                      int32_t decode_hint);

/* A probe of the kernels' bounded waits (no counterpart in the reference,
 * whose kernels are library calls): one warp waits on an mbarrier phase that
 * nothing completes and then polls *never_set (a device int32 that must stay
 * 0), each wait giving up after about 1 s as every wait in this library does;
 * both set PKV_DEV_WAIT_TIMEOUT in *dev_status, and *result (if non-NULL)
 * gets bit 0 / bit 1 set only if the barrier / the word were seen (0 when
 * both waits ran out). About 2 s of one warp on `stream`; the context stays
 * usable. For tests and health checks of a deployment. */
PKV_API int pkv_wait_probe(const int32_t* never_set, int32_t* dev_status, int32_t* result, void* stream);

/* Decode attention that allocates nothing and takes no workspace. No
 * counterpart in the reference: it is for callers that cannot allocate device
 * memory — a serving process that gives (nearly) all of HBM to its KV pool and
 * allocates nothing afterwards, or a host that owns every device allocation
 * and does not let a plug-in library call cudaMalloc. Same arguments and
 * result as pkv_attend with decode_hint = 1 (plan + split-K decode kernel), for
 * the decode kernel's geometry only (fp16/bf16 pool, head_dim 64, 16-token
 * pages, <= 8 KV heads, 1/2/4/8 query heads per KV head; PKV_ERR_UNSUPPORTED
 * otherwise).
 * Scratch: one file-scope 8 MiB device array, held by every GPU that loads
 * the library until the process exits; a batch needing more (about 340k pages
 * at 32 query heads, 190k at 64,
 * or very many sequences) is rejected with PKV_ERR_ARG. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture. Every call shares the array and leaves
 * its contents behind (each call re-initialises what it reads), so calls that
 * overlap on the GPU — on different streams, or from different threads —
 * race and must be serialised by the caller. Calls no cudaMalloc / cudaFree. */
PKV_API int pkv_attend_decode_noalloc(const pkv_pool* pool, int32_t layer, int32_t n_heads,
                                      const void* q, void* out, float scale,
                                      const pkv_batch* batch, void* stream);

/* ---- greedy sampling --------------------------------------------------------
 * Replaces the scheduler's torch.argmax(logits, dim=-1) after each forward pass
 * (serving/scheduler/scheduler.py:756-757); its .tolist() host read becomes the
 * caller's asynchronous copy of `sampled`, which can be read a step later.
 * For each of n_rows rows of `logits` (dtype PKV_F16 / PKV_BF16 / PKV_F32,
 * row r at logits + r * row_stride elements, `vocab` entries): the index of the
 * row maximum, the FIRST such index on ties, a NaN counting as larger than every
 * number (torch.argmax's result). The token is written to sampled[r] (int64,
 * if `sampled` is non-NULL) and to the token table: tokens[rows[r]] when `rows`
 * (int32 [n_rows]) is given — rows[r] < 0 skips the row, rows[r] >= tokens_len
 * skips it and sets PKV_DEV_SLOT_OOB in *dev_status — else tokens[r]. One launch
 * on `stream`; no workspace. */
PKV_API int pkv_sample_greedy(int32_t dtype, const void* logits, int64_t n_rows, int64_t vocab,
                              int64_t row_stride, const int32_t* rows, int64_t* tokens, int64_t tokens_len,
                              int64_t* sampled, int32_t* dev_status, void* stream);

/* ---- copy-on-write ---------------------------------------------------------
 * Replaces PagedTorchBackend.copy_block (serving/backends/paged_torch.py:181-207)
 * and FlashInferBackend.copy_block (flashinfer_backend.py:415-441), batched:
 * for every pair i, block dst[i] := block src[i] in every layer, K and V, in one
 * launch. src/dst: device int32 [n_pairs]. Pairs with src == dst are no-ops.
 * This function does NOT check that the destinations are distinct or that the
 * dst set is disjoint from the src set: the pairs run concurrently, so a chain
 * (a->b with b->c) or a repeated destination gives an order-dependent result.
 * The caller guarantees both (the Python wrapper B200PagedBackend.copy_blocks
 * checks them on the host before calling). Ids outside the pool are skipped and
 * flagged PKV_DEV_SLOT_OOB. */
PKV_API int pkv_copy_blocks(const pkv_pool* pool, const int32_t* src, const int32_t* dst,
                    int64_t n_pairs, int32_t* dev_status, void* stream);

/* The reference's exact signature, copy_block(src, dst), ids by value:
 * PKV_ERR_ARG when either id is outside [0, num_blocks) (the reference raises
 * IndexError, paged_torch.py:199-202); src == dst is a no-op. */
PKV_API int pkv_copy_block(const pkv_pool* pool, int64_t src, int64_t dst, void* stream);

/* ---- step descriptor assembly ---------------------------------------------
 * Replaces build_batch_meta (serving/engine_iface/batch.py:190-318) with
 * SequenceBlocks.slots_for_new_tokens (serving/memory/block_table.py:100-121)
 * and build_csr (block_table.py:184-208): the BatchMeta fields of one step are
 * computed on the device from a device-resident block table whose rows hold
 * each sequence's physical block ids in logical order. The host sends only the
 * step's rows and lengths plus the table entries that changed. */
typedef struct pkv_block_tables {
  int32_t* table;      /* device [max_seqs][max_pages]: row r = one sequence's block ids */
  int32_t max_seqs;
  int32_t max_pages;   /* entries per row */
  int32_t block_size;  /* tokens per page */
  int32_t reserved;
} pkv_block_tables;

/* Device outputs, the BatchMeta fields (docs/ARCHITECTURE.md:88-120). The
 * kernels write at most seqs_cap (+1 for the two prefix sums) / tokens_cap /
 * pages_cap entries of the respective arrays. */
typedef struct pkv_meta_out {
  int32_t* query_lens;       /* [n] */
  int32_t* cu_query_lens;    /* [n+1] exclusive prefix sum of query_lens */
  int32_t* kv_lens;          /* [n] */
  int64_t* positions;        /* [T] absolute positions kv_len-q_len .. kv_len-1 */
  int32_t* last_token_ix;    /* [n] cu_query_lens[i+1] - 1 */
  int32_t* kv_indptr;        /* [n+1] */
  int32_t* kv_indices;       /* [sum of ceil(kv_len / block_size)] table rows, page order */
  int32_t* kv_last_page_len; /* [n] in [1, block_size] */
  int32_t* batch_indices;    /* [T] owning sequence of each token */
  int32_t* slot_mapping;     /* [T] block * block_size + position % block_size */
  int32_t seqs_cap;
  int32_t reserved;
  int64_t tokens_cap;
  int64_t pages_cap;
} pkv_meta_out;

/* One step's BatchMeta. Input: int32 words rows[n] query_lens[n] kv_lens[n]
 * upd_row[u] upd_page[u] upd_block[u], in `step_dev` (device); if `step_host`
 * is non-NULL (pinned host memory) those 3n + 3u words are first copied from it
 * to `step_dev` on `stream`. On the device, in stream order: the u table writes
 * table[upd_row][upd_page] = upd_block, then every output field of the n
 * sequences (sequence i = table row rows[i], kv_len = kv_lens[i] AFTER this
 * step's append, query_len = query_lens[i]). PKV_ERR_ARG for an empty batch
 * (the reference raises ValueError, batch.py:238-242) or n > seqs_cap. On the
 * device, an update outside the table, a row outside it, query_len < 1,
 * query_len > kv_len, a page count above max_pages, or totals above the
 * capacities set PKV_DEV_META_BAD in *dev_status; such a sequence gets no
 * pages and slot -1 for its tokens. */
PKV_API int pkv_build_batch_meta(const pkv_block_tables* tables, const int32_t* step_host, int32_t* step_dev,
                                 int32_t n_seqs, int32_t n_updates, const pkv_meta_out* out,
                                 int32_t* dev_status, void* stream);

/* ---- swap gather / scatter ------------------------------------------------
 * Replace KVSwapSpace._to_host / _from_host (serving/scheduler/preemption.py:490-523).
 * Host layout of a swapped sequence (the SwapHandle's k / v,
 * preemption.py:303-333): [num_layers][nb][block_size][n_kv_heads][head_dim],
 * K and V in separate buffers, block i of the handle = block_ids[i].
 *
 * pkv_swap_gather:  staging[(kv*L + l)*nb + i] = pool block block_ids[i], layer l
 * pkv_swap_scatter: the reverse. `staging` is device memory holding the two
 * host buffers back to back (K then V): 2 * L * nb * block_bytes. */
PKV_API int pkv_swap_gather(const pkv_pool* pool, const int32_t* block_ids, int64_t nb, void* staging,
                    int32_t* dev_status, void* stream);
PKV_API int pkv_swap_scatter(const pkv_pool* pool, const int32_t* block_ids, int64_t nb,
                     const void* staging, int32_t* dev_status, void* stream);

/* Asynchronous swap engine: device gather into a bounded, double-buffered
 * staging area, copy-engine transfers to/from pinned host memory on a private
 * stream, events ordering it against the caller's compute stream. */
typedef struct pkv_swapper pkv_swapper;

/* `staging` (device) of `staging_bytes` is borrowed for the swapper's lifetime. */
PKV_API int pkv_swapper_create(void* staging, size_t staging_bytes, pkv_swapper** out);
PKV_API int pkv_swapper_destroy(pkv_swapper* sw);

/* Swap-out of one sequence: reads blocks block_ids[0..nb) (device int32) of every
 * layer into pinned host buffers host_k / host_v (each L*nb*block_bytes).
 * Ordering: starts after all work already queued on `compute_stream`; work queued
 * on `compute_stream` after this call starts only after the device has finished
 * READING the blocks, so the caller may free the blocks as soon as this returns.
 * The host buffers are complete once pkv_swapper_wait(sw, ticket) returns, where
 * *ticket is set to this operation's ticket. */
PKV_API int pkv_swap_out(pkv_swapper* sw, const pkv_pool* pool, const int32_t* block_ids, int64_t nb,
                 void* host_k, void* host_v, void* compute_stream, int32_t* dev_status,
                 uint64_t* ticket);

/* Swap-in: writes host_k / host_v into blocks block_ids[0..nb) of every layer.
 * Starts after work already queued on `compute_stream`; work queued on
 * `compute_stream` afterwards sees the restored blocks. The host buffers may be
 * released once pkv_swapper_wait(sw, ticket) returns. */
PKV_API int pkv_swap_in(pkv_swapper* sw, const pkv_pool* pool, const int32_t* block_ids, int64_t nb,
                const void* host_k, const void* host_v, void* compute_stream,
                int32_t* dev_status, uint64_t* ticket);

/* Block the host until operation `ticket` (0 = everything issued) completed. */
PKV_API int pkv_swapper_wait(pkv_swapper* sw, uint64_t ticket);
/* 1 if `ticket` completed, 0 if still in flight. */
PKV_API int pkv_swapper_done(pkv_swapper* sw, uint64_t ticket);

#ifdef __cplusplus
}
#endif

#endif /* PKV_H_ */
