// sffn_wait_probe: the library's two kinds of bounded wait -- an mbarrier
// wait (GEMM and pack pipelines) and a decoupled look-back (tile and flat
// packs) -- run on something that never happens, with a short limit the
// caller chooses, so that a test can check that a wait which runs out records
// SFFN_STATUS_WAIT_TIMEOUT in the status word and returns, leaving the context
// usable.  Nothing here faults: the mbarrier belongs to the kernel itself and
// has no copy in flight, and the look-back reads a zeroed state array.
#include "common.cuh"
#include "sm100.cuh"

namespace sffn {
namespace {

// Phase 0 of a barrier that nothing arrives on never completes.
__global__ void wait_probe_mbar_kernel(unsigned long long limit_ns, uint32_t* status,
                                       unsigned long long* elapsed) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer_ns();
        if (!mbar_wait_bounded(&bar, 0u, limit_ns)) atomicOr(status, SFFN_STATUS_WAIT_TIMEOUT);
        if (elapsed) *elapsed = globaltimer_ns() - t0;
    }
}

// Partition kProbePart looks back over predecessors that never publish.
constexpr long long kProbePart = 40;
__global__ void wait_probe_lookback_kernel(unsigned long long* states, unsigned long long limit_ns,
                                           uint32_t* status, unsigned long long* elapsed) {
    const int lane = threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    if (lane == 0) lookback_publish_relaxed(states, kProbePart, 7);
    __syncwarp();
    (void)lookback_rows<4>(states, kProbePart, 7, status, lane, limit_ns);
    if (lane == 0 && elapsed) *elapsed = globaltimer_ns() - t0;
}

}  // namespace
}  // namespace sffn

using namespace sffn;

extern "C" int sffn_wait_probe(int kind, int64_t limit_ns, uint64_t* states, uint64_t* elapsed_ns_dev,
                               uint32_t* status_dev, void* stream) {
    if (kind != 0 && kind != 1) return SFFN_ERR_ARG;
    if (limit_ns <= 0 || limit_ns > 100ll * 1000 * 1000 || !status_dev) return SFFN_ERR_ARG;
    if (kind == 1 && !states) return SFFN_ERR_ARG;
    DeviceScope dev_scope;
    if (int rc = dev_scope.bind_same(status_dev, {states, elapsed_ns_dev})) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (kind == 0) {
        wait_probe_mbar_kernel<<<1, 32, 0, st>>>((unsigned long long)limit_ns, status_dev,
                                                 reinterpret_cast<unsigned long long*>(elapsed_ns_dev));
    } else {
        SFFN_CUDA_TRY(cudaMemsetAsync(states, 0, 64 * sizeof(uint64_t), st));
        wait_probe_lookback_kernel<<<1, 32, 0, st>>>(reinterpret_cast<unsigned long long*>(states),
                                                     (unsigned long long)limit_ns, status_dev,
                                                     reinterpret_cast<unsigned long long*>(elapsed_ns_dev));
    }
    SFFN_CHECK_LAUNCH();
    return SFFN_OK;
}
