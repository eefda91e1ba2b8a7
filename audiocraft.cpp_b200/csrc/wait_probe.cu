// wait_probe.cu -- a kernel whose only job is to let a bounded device wait run out.
//
// Every wait in the tcgen05 kernels (mbarrier phases, the stream-K hand-off flag) gives up after
// a time limit, records a code in the context's device error word and returns, so that a wait
// which can never finish ends the kernel instead of hanging the GPU; the host reads the word
// after each step.  This kernel runs the same bounded flag wait on a flag that nothing sets, with
// a caller-chosen limit, so that tests can watch that path end in an error status on a live
// context without faulting or hanging anything.
#include "kernels.h"
#include "tc_common.cuh"

namespace act {

namespace {

__global__ void wait_probe_kernel(const int* flag, unsigned long long limit_ns, int* err) {
    if (threadIdx.x == 0 && blockIdx.x == 0) tc::flag_wait(flag, 1, err, WAIT_PROBE_CODE, limit_ns);
}

}  // namespace

void wait_probe(const int* flag, long long limit_ns, int* err, cudaStream_t s) {
    wait_probe_kernel<<<1, 32, 0, s>>>(flag, (unsigned long long)(limit_ns > 0 ? limit_ns : 1), err);
}

}  // namespace act
