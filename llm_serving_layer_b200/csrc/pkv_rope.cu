// pkv_rope.cu — rotary position embedding of q and k at each token's position.
//
// The engine rotates q and k at meta.positions before append_kv / attend
// (docs/ARCHITECTURE.md:167-172: project Q/K/V, RoPE, append, attend). For a
// decode batch the decode kernel does this itself (pkv_append_attend_rope_planned);
// this kernel serves every other batch (chunked prefill, mixed steps) and
// callers that want the rotation alone: one launch for q and k together, in
// place or into separate outputs.
//
// Each thread owns one pair (i, i + D/2) of one head of one token, reads the
// token's cosine / sine i from the caller's tables [max_pos][D/2] (fp32) and
// rounds as the fp32 elementwise formula a*cos - b*sin, a*sin + b*cos does
// (rope_pair), then to the pool dtype with round-to-nearest-even. A position
// outside [0, max_pos) leaves its pairs unrotated and sets PKV_DEV_META_BAD.
#include <algorithm>

#include "pkv_common.cuh"

namespace pkv {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const T* xq, T* yq, const T* xk, T* yk, int64_t n_tokens,
                                                   int hq, int hk, int half, const int64_t* positions,
                                                   const float* cs, const float* sn, int64_t max_pos,
                                                   int32_t* st) {
  pdl_trigger();
  pdl_wait();  // q, k and the positions may come from the kernels just before
  const int64_t per_tok = int64_t(hq + hk) * half;
  const int64_t total = n_tokens * per_tok;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t t = idx / per_tok;
    const int r = int(idx - t * per_tok);
    int hh = r / half;
    const int i = r - hh * half;
    const T* x;
    T* y;
    if (hh < hq) {
      x = xq + (t * hq + hh) * 2 * half;
      y = yq + (t * hq + hh) * 2 * half;
    } else {
      hh -= hq;
      x = xk + (t * hk + hh) * 2 * half;
      y = yk + (t * hk + hh) * 2 * half;
    }
    float a = to_f<T>(x[i]), b = to_f<T>(x[i + half]);
    const int64_t p = positions[t];
    if (p >= 0 && p < max_pos) {
      rope_pair(a, b, cs[p * half + i], sn[p * half + i]);
    } else if (i == 0) {
      flag(st, PKV_DEV_META_BAD);
    }
    y[i] = from_f<T>(a);
    y[i + half] = from_f<T>(b);
  }
}

template <typename T>
int launch_rope(const void* q, void* q_out, int32_t n_heads, const void* k, void* k_out, int32_t n_kv_heads,
                int64_t n_tokens, int32_t head_dim, const int64_t* positions, const float* cs, const float* sn,
                int64_t max_pos, int32_t* st, cudaStream_t s) {
  const int half = head_dim / 2;
  const int64_t total = n_tokens * int64_t(n_heads + n_kv_heads) * half;
  const int64_t want = (total + 255) / 256;
  const int grid = int(std::min<int64_t>(want, int64_t(8) * num_sms()));
  PKV_CUDA_RET(launch_kernel(rope_kernel<T>, dim3(grid), dim3(256), 0, s, true, static_cast<const T*>(q),
                             static_cast<T*>(q_out), static_cast<const T*>(k), static_cast<T*>(k_out), n_tokens,
                             int(n_heads), int(n_kv_heads), half, positions, cs, sn, max_pos, st));
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_rope(int32_t dtype, const void* q, void* q_out, int32_t n_heads, const void* k, void* k_out,
                        int32_t n_kv_heads, int64_t n_tokens, int32_t head_dim, const int64_t* positions,
                        const float* rope_cos, const float* rope_sin, int64_t rope_max_pos, int32_t* dev_status,
                        void* stream) {
  if (dtype != PKV_F16 && dtype != PKV_BF16) return fail(PKV_ERR_UNSUPPORTED, "pkv_rope takes fp16 or bf16");
  if (n_tokens < 0 || n_heads < 0 || n_kv_heads < 0)
    return fail(PKV_ERR_ARG, "n_tokens, n_heads and n_kv_heads must be >= 0");
  if (head_dim <= 0 || head_dim % 2 || head_dim > 1024)
    return fail(PKV_ERR_ARG, "head_dim must be even and in [2, 1024]");
  if (n_heads > 0 && (!q || !q_out)) return fail(PKV_ERR_ARG, "q and q_out must be non-NULL when n_heads > 0");
  if (n_kv_heads > 0 && (!k || !k_out))
    return fail(PKV_ERR_ARG, "k and k_out must be non-NULL when n_kv_heads > 0");
  if (n_tokens == 0 || n_heads + n_kv_heads == 0) return PKV_OK;
  if (!positions || !rope_cos || !rope_sin)
    return fail(PKV_ERR_ARG, "positions, rope_cos and rope_sin must be non-NULL");
  if (rope_max_pos <= 0) return fail(PKV_ERR_ARG, "rope_max_pos must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PKV_F16)
    return launch_rope<__half>(q, q_out, n_heads, k, k_out, n_kv_heads, n_tokens, head_dim, positions, rope_cos,
                               rope_sin, rope_max_pos, dev_status, s);
  return launch_rope<__nv_bfloat16>(q, q_out, n_heads, k, k_out, n_kv_heads, n_tokens, head_dim, positions,
                                    rope_cos, rope_sin, rope_max_pos, dev_status, s);
}
