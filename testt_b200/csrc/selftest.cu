// Self-test of the bounded mbarrier wait that every waiting kernel of the library uses (the
// tensor-core GEMMs' pipelines): a wait whose phase never completes gives up after its poll
// limit, counts itself in the device's timeout counter (tb_wait_timeouts) and lets the kernel
// return with an error status, so the CUDA context stays usable. Only an mbarrier in this
// CTA's own shared memory is waited on; nothing else is touched.
#include "common.cuh"

namespace tb {
namespace {

// One thread initialises an mbarrier expecting one arrival, arrives on it or not, and waits on
// phase 0 for at most `polls` polls; status = 0 when the phase completed, 1 when it gave up.
__global__ void wait_selftest_kernel(uint32_t polls, int arrive, int32_t *status) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_init_fence();
  if (arrive) mbar_arrive(&bar);
  const bool done = mbar_wait(&bar, 0, polls);
  if (!done) atomicAdd(&g_wait_timeouts, 1u);
  *status = done ? 0 : 1;
}

}  // namespace

TB_REGISTER_TIMEOUT_READER(selftest)

}  // namespace tb

using namespace tb;

extern "C" int tb_wait_selftest(int32_t polls, int32_t arrive, int32_t *status, void *stream) {
  if (polls <= 0 || status == nullptr)
    return set_error(TB_EINVAL, "wait_selftest: polls %d (> 0) and a status buffer", polls);
  wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>((uint32_t)polls, arrive != 0, status);
  note_launch();
  return check_launch("wait_selftest");
}
