// SM clock measured from inside the GPU: one thread counts SM cycles against
// the global nanosecond timer over a short window.  No counterpart in the
// reference; it lets a benchmark record the clock under load without a
// driver query (NVML or nvidia-smi), which stalls the host's synchronisations.
#include "common.cuh"

namespace zmoe {
namespace {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// out[0] = SM cycles, out[1] = nanoseconds elapsed over the window.  The loop
// ends after window_ns or a fixed number of polls, whichever comes first.
__global__ void clock_probe_kernel(uint64_t* out, uint64_t window_ns) {
  const uint64_t t0 = global_ns();
  const long long c0 = clock64();
  uint64_t t1 = t0;
  long long c1 = c0;
  for (uint32_t it = 0; it < (1u << 24) && t1 - t0 < window_ns; ++it) {
    t1 = global_ns();
    c1 = clock64();
  }
  out[0] = (uint64_t)(c1 - c0);
  out[1] = t1 - t0;
}

}  // namespace
}  // namespace zmoe

extern "C" zmoe_status zmoe_clock_probe(uint64_t* out, uint64_t window_ns, zmoe_stream_t stream) {
  ZMOE_CHECK_ARG(out, "clock_probe: null pointer");
  ZMOE_CHECK_ARG(window_ns > 0 && window_ns <= 10000000ull, "clock_probe: window %llu ns outside (0, 10 ms]",
                 (unsigned long long)window_ns);
  zmoe::clock_probe_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(out, window_ns);
  return zmoe::launch_status("clock_probe_kernel");
}
