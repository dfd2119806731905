// Grouped expert FFN for callers that cannot allocate device memory.
//
// zmoe_expert_ffn needs a BF16 scratch buffer h of rows_total * I elements for
// the SwiGLU / ReLU intermediate, which its caller must cudaMalloc.  Some
// callers cannot: a serving runtime that owns all device memory through its
// own pool and forbids plugins from calling cudaMalloc/cudaFree (a cudaFree
// synchronises the whole device and would stall every stream it runs), or code
// that must not touch the allocator in the middle of a step.  This entry point
// takes the same inputs and outputs and keeps the intermediate in a file-scope
// device array instead, so it calls no cudaMalloc, cudaFree or allocating
// library routine.
//
// Limits and sharing:
//  * the array holds kNoAllocScratchElems BF16 values (32 MiB); a call whose
//    rows_total * I exceeds that is rejected with ZMOE_EUNSUPPORTED;
//  * every GPU that loads the library holds the array until the process exits;
//  * all calls share the array and it keeps the last call's contents; nothing
//    in it needs to start at zero (every element read was written by the same
//    call first);
//  * calls that overlap on the GPU (two streams, or two host threads) race on
//    the array and give wrong results: serialise them;
//  * the first call on a device looks up the array's device address with that
//    device current (cudaGetSymbolAddress); make that first call before any
//    stream capture.
#include <mutex>

#include "common.cuh"

namespace zmoe {


namespace {

constexpr size_t kNoAllocScratchElems = 16u << 20;   // BF16 elements = 32 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint16_t g_ffn_scratch[kNoAllocScratchElems];

std::mutex g_mu;
uint16_t* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_ffn_scratch on the current device (looked up once per device).
zmoe_status scratch_for_current_device(uint16_t** out) {
  int dev = -1;
  ZMOE_CUDA_RET(cudaGetDevice(&dev));
  ZMOE_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "expert_ffn_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    ZMOE_CUDA_RET(cudaGetSymbolAddress(&p, g_ffn_scratch));
    g_scratch_ptr[dev] = static_cast<uint16_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return ZMOE_OK;
}

}  // namespace
}  // namespace zmoe

extern "C" zmoe_status zmoe_expert_ffn_noalloc(const zmoe_ffn_args* a, zmoe_stream_t stream) {
  ZMOE_CHECK_ARG(a && a->x && a->w && a->y, "expert_ffn_noalloc: null pointer");
  ZMOE_CHECK_ARG(a->I > 0 && a->rows_total >= 0, "expert_ffn_noalloc: bad sizes");
  const size_t need = (size_t)(a->rows_total > 0 ? a->rows_total : 0) * (size_t)a->I;
  if (need > zmoe::kNoAllocScratchElems) {
    zmoe::set_error("expert_ffn_noalloc: rows_total*I = %zu exceeds the %zu-element scratch; "
                    "use zmoe_expert_ffn with a caller buffer", need, zmoe::kNoAllocScratchElems);
    return ZMOE_EUNSUPPORTED;
  }
  uint16_t* scratch = nullptr;
  zmoe_status st = zmoe::scratch_for_current_device(&scratch);
  if (st != ZMOE_OK) return st;
  zmoe_ffn_args b = *a;
  b.h = scratch;
  return zmoe::launch_expert_ffn(&b, reinterpret_cast<cudaStream_t>(stream));
}
