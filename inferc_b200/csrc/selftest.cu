// Self-test of the bounded-wait failure path, without a GPU fault.
//
// Every wait in this library's kernels (mbarrier phases of the TMA /
// tcgen05 pipelines, grid barriers of the persistent decode kernel) gives up
// after a time limit, sets a device error flag and lets its CTA leave; the
// host then reports INFERC_ERR_TIMEOUT from inferc_dev_stream_synchronize and
// the context stays usable. This file runs those wait loops on something that
// is never signalled (an mbarrier nothing arrives at, an arrival counter no
// CTA increments) with a caller-chosen short limit, so a test can watch the
// whole path: the wait gives up, the flag is set, the host reads and clears
// it, and later launches work. Nothing here traps, faults or spins without a
// bound.
#include "tc_ptx.cuh"

namespace inferc_dev {
namespace {

__device__ int g_selftest_error;

__global__ void selftest_mbar_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0 && !tc::mbar_wait(&bar, 0, limit_ns)) atomicExch(&g_selftest_error, 1);
  __syncthreads();
}

// The grid-barrier wait of the persistent decode kernel: thread 0 polls an
// arrival counter with acquire loads until it reaches its target, giving up
// after limit_ns (checked every 64 polls) or when another CTA flagged an error.
__global__ void selftest_grid_kernel(unsigned int* counter, unsigned long long limit_ns) {
  if (threadIdx.x == 0) {
    const unsigned target = gridDim.x + 1;  // one more arrival than CTAs exist
    atomicAdd(counter, 1u);
    const unsigned long long t0 = tc::gclock_ns();
    for (uint32_t i = 0;;) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if ((int)(v - target) >= 0) break;
      if ((++i & 63) == 0 &&
          (tc::gclock_ns() - t0 > limit_ns || *(volatile int*)&g_selftest_error)) {
        atomicExch(&g_selftest_error, 1);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace

int read_and_clear_selftest_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_selftest_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_selftest_error, &z, sizeof(int)));
  }
  return v;
}

}  // namespace inferc_dev

extern "C" int inferc_dev_selftest_wait_timeout(int which, int64_t limit_us, void* stream) {
  using namespace inferc_dev;
  return guard([&] {
    IDEV_CHECK_ARG(which == 0 || which == 1, "selftest: which must be 0 (mbarrier) or 1 (grid)");
    IDEV_CHECK_ARG(limit_us >= 1 && limit_us <= 1000000, "selftest: limit must be in [1us, 1s]");
    cudaStream_t st = as_stream(stream);
    const unsigned long long ns = (unsigned long long)limit_us * 1000ull;
    if (which == 0) {
      selftest_mbar_kernel<<<1, 32, 0, st>>>(ns);
      IDEV_LAUNCHED();
    } else {
      void* counter = nullptr;
      IDEV_CUDA(cudaMallocAsync(&counter, sizeof(unsigned int), st));
      IDEV_CUDA(cudaMemsetAsync(counter, 0, sizeof(unsigned int), st));
      selftest_grid_kernel<<<4, 32, 0, st>>>(static_cast<unsigned int*>(counter), ns);
      IDEV_LAUNCHED();
      IDEV_CUDA(cudaFreeAsync(counter, st));
    }
  });
}
