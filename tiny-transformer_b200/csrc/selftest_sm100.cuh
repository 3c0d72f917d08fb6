// Diagnostic kernel for the failure path of the bounded waits: one warp waits on an mbarrier
// phase that nothing completes, with a short cycle budget. The wait must give up on its own,
// record TT_ERR_TIMEOUT in the device status word and return, leaving the CUDA context usable.
// It runs the same mbar_wait used by the attention kernels; it issues no TMA, allocates no
// TMEM and touches no global memory other than the status word.
#pragma once

#include "sm100_ptx.cuh"

namespace tt {
namespace selftest {

// Upper bound accepted by the host entry point (~0.5 s at 1.9 GHz).
constexpr long long kMaxSelftestBudget = 1000000000LL;

__global__ void __launch_bounds__(32, 1) wait_timeout_kernel(long long budget_cycles) {
  __shared__ alignas(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival, which never comes
    fence_barrier_init();
  }
  __syncwarp();
  mbar_wait(&bar, 0, budget_cycles);
}

}  // namespace selftest
}  // namespace tt
