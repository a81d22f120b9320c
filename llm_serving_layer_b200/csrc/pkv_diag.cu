// pkv_diag.cu — a probe of the kernels' bounded waits.
//
// Every wait in this library's kernels (on an mbarrier phase: TMA data, a ring
// slot, a handoff; on a word another warp or CTA sets) gives up after about a
// second of %globaltimer, records PKV_DEV_WAIT_TIMEOUT in the caller's status
// word and lets the kernel unwind, so a missing arrival becomes an error the
// host reads instead of a hung GPU. This probe makes both kinds of wait run
// out on purpose: one warp waits, through the same helper the kernels use, on
// an mbarrier phase that nothing completes, then polls a device word that
// nothing sets, with the loop the decode kernel uses for its merge handoffs.
// No copy is in flight and nothing else is touched, so the context stays
// usable afterwards.
#include "pkv_common.cuh"

namespace pkv {
namespace {

__global__ void __launch_bounds__(32) wait_probe_kernel(const int32_t* never_set, int32_t* st, int32_t* result) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival completes phase 0; none comes
    fence_mbar_init();
  }
  __syncthreads();
  const bool got_bar = mbar_wait_bounded(&bar, 0, st);
  int got_word = 0;
  if (threadIdx.x == 0) {
    const volatile int32_t* f = never_set;
    const uint64_t t0 = globaltimer_ns();
    while (!(got_word = *f) && globaltimer_ns() - t0 < 1000000000ull) __nanosleep(64);
    if (!got_word) flag(st, PKV_DEV_WAIT_TIMEOUT);
    if (result) *result = (got_bar ? 1 : 0) | (got_word ? 2 : 0);
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_wait_probe(const int32_t* never_set, int32_t* dev_status, int32_t* result, void* stream) {
  if (!never_set || !dev_status) return fail(PKV_ERR_ARG, "never_set and dev_status must be non-NULL");
  PKV_CUDA_RET(launch_kernel(wait_probe_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), false,
                             never_set, dev_status, result));
  PKV_CUDA_RET(cudaGetLastError());
  return PKV_OK;
}
