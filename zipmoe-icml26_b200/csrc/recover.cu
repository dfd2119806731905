// Plane recombine (replaces cuda_recover_uint16_to_bf16,
// csrc/kernels/tensor_recover.cu:12-43, launcher :47-63).
//
// The reference kernel moves 8 elements per thread with 64-bit accesses and a
// 32-bit element count.  This one moves 16 elements per thread per step with
// 128-bit loads of both planes and two 128-bit stores, spreads the bytes into
// 16-bit lanes with byte permutes, and runs a grid-stride loop over a 64-bit
// count sized to the 148 SMs.
#include "common.cuh"

namespace zmoe {
namespace {

__device__ __forceinline__ uint32_t recombine2(uint32_t e_bytes, uint32_t s_bytes, uint32_t sel) {
  // e_bytes/s_bytes hold 4 bytes; sel picks two of them into 16-bit lanes.
  const uint32_t e2 = __byte_perm(e_bytes, 0, sel);
  const uint32_t s2 = __byte_perm(s_bytes, 0, sel);
  return ((s2 & 0x00800080u) << 8) | (e2 << 7) | (s2 & 0x007F007Fu);
}

__global__ void __launch_bounds__(256)
recover_vec_kernel(uint4* __restrict__ out, const uint4* __restrict__ exp, const uint4* __restrict__ sm,
                   size_t n16) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 e = __ldg(exp + i);
    const uint4 s = __ldg(sm + i);
    uint4 lo, hi;
    lo.x = recombine2(e.x, s.x, 0x4140);
    lo.y = recombine2(e.x, s.x, 0x4342);
    lo.z = recombine2(e.y, s.y, 0x4140);
    lo.w = recombine2(e.y, s.y, 0x4342);
    hi.x = recombine2(e.z, s.z, 0x4140);
    hi.y = recombine2(e.z, s.z, 0x4342);
    hi.z = recombine2(e.w, s.w, 0x4140);
    hi.w = recombine2(e.w, s.w, 0x4342);
    out[2 * i] = lo;
    out[2 * i + 1] = hi;
  }
}

__global__ void __launch_bounds__(256)
recover_scalar_kernel(uint16_t* __restrict__ out, const uint8_t* __restrict__ exp,
                      const uint8_t* __restrict__ sm, size_t begin, size_t n) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = begin + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = (uint16_t)recombine(sm[i], exp[i]);
}

}  // namespace

zmoe_status launch_tensor_recover(uint16_t* out, const uint8_t* exp, const uint8_t* sm, size_t n,
                                  cudaStream_t stream) {
  if (n == 0) return ZMOE_OK;
  const bool aligned = ((uintptr_t)out % 16 == 0) && ((uintptr_t)exp % 16 == 0) && ((uintptr_t)sm % 16 == 0);
  size_t done = 0;
  if (aligned && n >= 16) {
    const size_t n16 = n / 16;
    size_t blocks = (n16 + 255) / 256;
    const size_t cap = (size_t)kNumSMs * 8;
    if (blocks > cap) blocks = cap;
    recover_vec_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
        reinterpret_cast<uint4*>(out), reinterpret_cast<const uint4*>(exp),
        reinterpret_cast<const uint4*>(sm), n16);
    zmoe_status st = launch_status("recover_vec_kernel");
    if (st != ZMOE_OK) return st;
    done = n16 * 16;
  }
  if (done < n) {
    size_t blocks = (n - done + 255) / 256;
    const size_t cap = (size_t)kNumSMs * 8;
    if (blocks > cap) blocks = cap;
    recover_scalar_kernel<<<(unsigned)blocks, 256, 0, stream>>>(out, exp, sm, done, n);
    return launch_status("recover_scalar_kernel");
  }
  return ZMOE_OK;
}

}  // namespace zmoe
