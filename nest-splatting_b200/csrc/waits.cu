// waits.cu -- self-test of the bounded waits.
//
// Every wait of this library's kernels on a word another CTA publishes (the
// radix sort's decoupled look-back) or on a barrier (the blend's record ring)
// gives up after a poll bound (ns_set_wait_limit), records an error bit in a
// device status word and lets the kernel finish, so a stalled producer can
// never hang the GPU. This kernel runs the same wait (wait_word) on a caller's
// word, for tests of that path: with a word that nothing sets, the wait must
// run out, set kErrSpinTimeout and return.
#include "kernels.cuh"

namespace ns {
namespace {

__global__ void wait_selftest_kernel(const uint32_t* flag, uint32_t limit, uint32_t* err) {
  if (threadIdx.x == 0 && wait_word(flag, 0xffffffffu, limit) == 0u) set_error(err, kErrSpinTimeout);
}

}  // namespace

int wait_selftest_launch(const uint32_t* flag, uint32_t* err, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(flag, ns_host::wait_limit(), err);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
