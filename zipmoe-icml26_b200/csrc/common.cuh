// Shared helpers for the sm_100a kernels and the C ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/zmoe.h"

namespace zmoe {

// Last error text of the calling host thread (zmoe_last_error()).
void set_error(const char* fmt, ...);

#define ZMOE_CHECK_ARG(cond, ...)              \
  do {                                         \
    if (!(cond)) {                             \
      ::zmoe::set_error(__VA_ARGS__);          \
      return ZMOE_EINVAL;                      \
    }                                          \
  } while (0)

#define ZMOE_CUDA_RET(expr)                                                      \
  do {                                                                           \
    cudaError_t e_ = (expr);                                                     \
    if (e_ != cudaSuccess) {                                                     \
      ::zmoe::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),  \
                        __FILE__, __LINE__);                                     \
      return ZMOE_ECUDA;                                                         \
    }                                                                            \
  } while (0)

inline zmoe_status launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return ZMOE_ECUDA;
  }
  return ZMOE_OK;
}

constexpr int kNumSMs = 148;

// Grouped expert FFN (ffn_tc.cu).  err: optional device word that a kernel
// whose bounded wait ran out sets to 1.
zmoe_status launch_expert_ffn(const zmoe_ffn_args* a, cudaStream_t stream, int32_t* err = nullptr);
// Device-wide error word of the FFN kernels on the current device.
zmoe_status read_kernel_error(int32_t* out, int reset);
// Error-path test hook: wait limit (cycles, <= 0 restores the default) and
// whether the FFN's TMA producer issues nothing.
void set_ffn_wait(long long cycles, int drop_loads);

// BF16 bit pattern from a sign+mantissa byte and an exponent byte
// (csrc/kernels/tensor_recover.cu:25-30).
__device__ __forceinline__ uint32_t recombine(uint32_t sm, uint32_t e) {
  return ((sm >> 7) << 15) | (e << 7) | (sm & 0x7Fu);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
  return __uint_as_float(b << 16);
}

__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}

// exp(x) for x <= 0 without fused multiply-add: Cody-Waite reduction with a
// two-part ln 2 (the high part has 15 significant bits, so n*LN2_HI is exact),
// then the degree-7 Taylor series of e^r in Horner form.  The same fp32
// operation sequence runs in the oracle, so results agree bit for bit.
__device__ __forceinline__ float exp_poly(float x) {
  // fp32 constants spelled as exact hexadecimal literals
  const float kLog2e = 0x1.715476p+0f;
  const float kLn2Hi = 0x1.62e4p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  if (x < -87.0f) return 0.0f;
  float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fsub_rn(x, __fmul_rn(n, kLn2Hi));
  r = __fsub_rn(r, __fmul_rn(n, kLn2Lo));
  float p = 0x1.a01a02p-13f;                      // 1/7!
  p = __fadd_rn(__fmul_rn(p, r), 0x1.6c16c2p-10f);  // 1/6!
  p = __fadd_rn(__fmul_rn(p, r), 0x1.111112p-7f);   // 1/5!
  p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-5f);   // 1/4!
  p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-3f);   // 1/3!
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  return ldexpf(p, (int)n);
}

}  // namespace zmoe
