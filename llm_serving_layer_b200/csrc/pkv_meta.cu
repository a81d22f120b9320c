// pkv_meta.cu — a step's BatchMeta assembled on the device from device-resident
// block tables.
//
// The reference assembles the step descriptor on the host every step
// (build_batch_meta, serving/engine_iface/batch.py:190-318): per sequence it
// extends Python lists with the absolute positions K-q..K-1, the owning
// sequence of each token, the slot of each new token
// (SequenceBlocks.slots_for_new_tokens via slot_for: slot = block_ids[p // P] * P + p % P,
// serving/memory/block_table.py:100-121), the exclusive prefix sum of the query
// lengths and the index of each sequence's last token; build_csr
// (block_table.py:184-208) concatenates the block ids into the CSR page table
// with kv_last_page_len in [1, P]; every field is then copied to the device.
//
// Here each sequence's block ids live in a row of a device table
// [max_seqs][max_pages] that the host updates incrementally (only ids that
// changed since the last step travel, as (row, page, block) triples in the same
// packed input as the step's rows / query lengths / kv lengths). Two kernels:
//   meta_scan_kernel  (one CTA): applies the table writes, then block-wide
//       exclusive scans of the query lengths and page counts -> cu_query_lens,
//       kv_indptr, and the per-sequence fields;
//   meta_fill_kernel  (a warp per sequence): copies the row's page ids into
//       kv_indices and writes positions, batch_indices and slot_mapping of the
//       sequence's new tokens. Launched with PDL after the scan kernel; it
//       waits for it before reading.
// A sequence whose row, lengths or page count are invalid (which the host
// wrapper rejects before launching) gets no pages, slot -1 for its tokens and
// PKV_DEV_META_BAD; the attention / append kernels then flag it again instead
// of reading through it. Every write is bounded by the output capacities.
#include "pkv_common.cuh"

namespace pkv {
namespace {

struct MetaIn {
  const int32_t* rows;
  const int32_t* ql;
  const int32_t* kv;
  const int32_t* upd_row;
  const int32_t* upd_page;
  const int32_t* upd_block;
  int32_t n;
  int32_t nu;
};

struct Tables {
  int32_t* table;
  int32_t max_seqs, max_pages, page;
};

// Pages of a valid sequence, or -1 when its row / lengths / page count are invalid.
__device__ __forceinline__ int seq_pages(const Tables& t, int row, int q, int k) {
  if (row < 0 || row >= t.max_seqs || q < 1 || k < q) return -1;
  const int pages = (k - 1) / t.page + 1;
  return pages <= t.max_pages ? pages : -1;
}

__global__ void __launch_bounds__(1024) meta_scan_kernel(Tables t, MetaIn in, pkv_meta_out o, int32_t* st) {
  __shared__ int warp_sum[32];
  pdl_trigger();  // the fill kernel may be scheduled now; it waits for this grid before reading
  for (int u = threadIdx.x; u < in.nu; u += blockDim.x) {
    const int r = in.upd_row[u], p = in.upd_page[u];
    if (r < 0 || r >= t.max_seqs || p < 0 || p >= t.max_pages) {
      flag(st, PKV_DEV_META_BAD);
      continue;
    }
    t.table[size_t(r) * t.max_pages + p] = in.upd_block[u];
  }
  int64_t carry_q = 0, carry_p = 0;
  for (int base = 0; base < in.n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool live = i < in.n;
    int q = 0, k = 0, pages = 0;
    if (live) {
      q = in.ql[i];
      k = in.kv[i];
      pages = seq_pages(t, in.rows[i], q, k);
      if (pages < 0) {
        flag(st, PKV_DEV_META_BAD);
        pages = 0;
      }
    }
    const int qs = q > 0 ? q : 0;
    int tot_q, tot_p;
    const int ex_q = block_excl_scan(qs, warp_sum, &tot_q);
    const int ex_p = block_excl_scan(pages, warp_sum, &tot_p);
    if (live) {
      const int64_t cq = carry_q + ex_q;
      o.query_lens[i] = q;
      o.kv_lens[i] = k;
      o.cu_query_lens[i] = int32_t(cq);
      o.last_token_ix[i] = int32_t(cq + qs - 1);
      o.kv_indptr[i] = int32_t(carry_p + ex_p);
      o.kv_last_page_len[i] = pages ? k - (pages - 1) * t.page : 0;
    }
    carry_q += tot_q;
    carry_p += tot_p;
  }
  if (threadIdx.x == 0) {
    o.cu_query_lens[in.n] = int32_t(carry_q);
    o.kv_indptr[in.n] = int32_t(carry_p);
    if (carry_q > o.tokens_cap || carry_p > o.pages_cap) flag(st, PKV_DEV_META_BAD);
  }
}

__global__ void __launch_bounds__(256) meta_fill_kernel(Tables t, MetaIn in, pkv_meta_out o) {
  pdl_wait();  // cu_query_lens / kv_indptr and the table writes of the scan kernel
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < in.n; i += warps) {
    const int row = in.rows[i], q = in.ql[i], k = in.kv[i];
    const int pages = seq_pages(t, row, q, k);
    const int64_t t0 = o.cu_query_lens[i], p0 = o.kv_indptr[i];
    const int32_t* trow = pages > 0 ? t.table + size_t(row) * t.max_pages : nullptr;
    for (int p = lane; p < pages; p += 32)
      if (p0 + p < o.pages_cap) o.kv_indices[p0 + p] = trow[p];
    for (int j = lane; j < q; j += 32) {
      const int64_t tok = t0 + j;
      if (tok >= o.tokens_cap) break;
      const int pos = k - q + j;
      o.positions[tok] = pos;
      o.batch_indices[tok] = i;
      o.slot_mapping[tok] = trow ? trow[pos / t.page] * t.page + pos % t.page : -1;
    }
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_build_batch_meta(const pkv_block_tables* tables, const int32_t* step_host, int32_t* step_dev,
                                    int32_t n_seqs, int32_t n_updates, const pkv_meta_out* out,
                                    int32_t* dev_status, void* stream) {
  if (!tables || !tables->table) return fail(PKV_ERR_ARG, "block tables must be non-NULL");
  if (tables->max_seqs <= 0 || tables->max_pages <= 0 || tables->block_size <= 0)
    return fail(PKV_ERR_ARG, "block tables need positive max_seqs, max_pages and block_size");
  if (n_seqs <= 0)
    return fail(PKV_ERR_ARG, "build_batch_meta() called with an empty sequence list");
  if (n_updates < 0) return fail(PKV_ERR_ARG, "n_updates must be >= 0");
  if (!step_dev) return fail(PKV_ERR_ARG, "step_dev must be non-NULL");
  if (!out || !out->query_lens || !out->cu_query_lens || !out->kv_lens || !out->positions ||
      !out->last_token_ix || !out->kv_indptr || !out->kv_indices || !out->kv_last_page_len ||
      !out->batch_indices || !out->slot_mapping)
    return fail(PKV_ERR_ARG, "every output field must be non-NULL");
  if (n_seqs > out->seqs_cap)
    return fail(PKV_ERR_ARG, std::to_string(n_seqs) + " sequences exceed the output capacity of " +
                                 std::to_string(out->seqs_cap));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t words = 3 * size_t(n_seqs) + 3 * size_t(n_updates);
  if (step_host) PKV_CUDA_RET(cudaMemcpyAsync(step_dev, step_host, words * 4, cudaMemcpyHostToDevice, s));
  const Tables t{tables->table, tables->max_seqs, tables->max_pages, tables->block_size};
  const int32_t* d = step_dev;
  const MetaIn in{d, d + n_seqs, d + 2 * size_t(n_seqs), d + 3 * size_t(n_seqs),
                  d + 3 * size_t(n_seqs) + n_updates, d + 3 * size_t(n_seqs) + 2 * size_t(n_updates),
                  n_seqs, n_updates};
  PKV_CUDA_RET(launch_kernel(meta_scan_kernel, dim3(1), dim3(1024), 0, s, false, t, in, *out, dev_status));
  const int warps_per_cta = 8;
  const int ctas = std::min((n_seqs + warps_per_cta - 1) / warps_per_cta, 4 * num_sms());
  PKV_CUDA_RET(launch_kernel(meta_fill_kernel, dim3(ctas), dim3(256), 0, s, true, t, in, *out));
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}
