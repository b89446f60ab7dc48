// Self-test of the bounded waits every pipelined kernel here relies on: each
// of the four wait helpers waits on an mbarrier that nothing ever arrives on,
// gives up after its time bound (2 s of %globaltimer) and records its own bit
// in the caller's result word.  Nothing faults or hangs: the kernel returns,
// and the context stays usable for the next launch.
#include "cb_async.cuh"
#include "cb_common.cuh"
#include "cb_tcgen05.cuh"

namespace {

__global__ void __launch_bounds__(128, 1) wait_selftest_kernel(int32_t* result) {
  __shared__ uint64_t bars[4];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) cb::tc::mbar_init(&bars[i], 1);  // one arrival that never comes
    cb::async::mbar_init_fence();
  }
  __syncthreads();
  bool ok = true;
  switch (warp) {
    case 0:  // single thread, suspend-hinted (tcgen05 kernels' producers and MMA issuers)
      if (lane == 0) ok = cb::tc::wait1(&bars[0], 0);
      break;
    case 1:  // whole warp, suspend-hinted (tcgen05 kernels' softmax / epilogue warps)
      ok = cb::tc::wait_warp(&bars[1], 0);
      break;
    case 2:  // whole warp (copy kernels' consumers)
      ok = cb::async::mbar_wait(&bars[2], 0);
      break;
    default:  // single thread (copy kernels' producers)
      if (lane == 0) ok = cb::async::mbar_wait_one(&bars[3], 0);
      break;
  }
  if (!ok && lane == 0) atomicOr(result, 1 << warp);
}

}  // namespace

extern "C" int cb_wait_selftest(int32_t* result, void* stream) {
  CB_BIND(stream, result);
  CB_REQUIRE(result != nullptr, "null result word");
  wait_selftest_kernel<<<1, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(result);
  return cb::launch_status("cb_wait_selftest");
}
