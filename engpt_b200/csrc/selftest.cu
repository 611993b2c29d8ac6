// Self-test of the bounded device-side wait (mbar_wait_limit), the failure
// path every tcgen05 kernel of this library relies on: a wait whose phase
// never completes gives up after its limit, records ENGPT_ERR_TIMEOUT with its
// site in the device status word, raises the CTA's abort word so the CTA's
// other waiting roles leave too, and the kernel returns normally.  Nothing
// faults or traps, so the context stays usable for the next launch.
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace engpt {
namespace selftest {

using namespace sm100;

constexpr int kSite = 99;        // site recorded by the wait that runs out
constexpr int kSiteFollow = 98;  // site of the second role's wait (it must leave through the abort word)

// Warp 0, lane 0 waits (with the given limit) on an mbarrier that nothing arrives on.  Warp 1, lane 0 waits on a
// second such barrier with the library's normal limit: it can only leave early through the CTA abort word the
// first wait raises when it runs out.  out[0] = 1 if the first wait reported failure, out[1] = 1 if the second did.
__global__ void wait_timeout_kernel(uint64_t limit_ns, int* out) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (lane == 0 && warp == 0) {
    const bool ok = mbar_wait_limit(smem_u32(&bars[0]), 0, abort_flag, kSite, limit_ns);
    out[0] = ok ? 0 : 1;
  } else if (lane == 0 && warp == 1) {
    const bool ok = mbar_wait(smem_u32(&bars[1]), 0, abort_flag, kSiteFollow);
    out[1] = ok ? 0 : 1;
  }
  __syncthreads();
}

}  // namespace selftest
}  // namespace engpt

using namespace engpt;

extern "C" int engpt_selftest_wait_timeout(int64_t limit_ns, int* flags_out, void* stream) {
  clear_error();
  ENGPT_REQUIRE(limit_ns > 0 && limit_ns <= 1000000000LL, ENGPT_ERR_ARG,
                "selftest_wait_timeout: limit %lld ns outside (0, 1 s]", (long long)limit_ns);
  ENGPT_REQUIRE(flags_out != nullptr, ENGPT_ERR_ARG, "selftest_wait_timeout: null output");
  selftest::wait_timeout_kernel<<<1, 64, 0, as_stream(stream)>>>((uint64_t)limit_ns, flags_out);
  return check_launch("selftest_wait_timeout");
}
