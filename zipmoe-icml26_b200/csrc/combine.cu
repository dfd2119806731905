// Combine (K5): gate-weighted sum of expert rows plus the shared expert.
//
// Replaces the per-expert Python loops of customized/qwen.py:89-100,
// customized/deepseek.py:103-115 and customized/switch_transformers.py:83-87,
// which accumulate into a BF16 buffer in completion order.  Here each thread
// owns 4 consecutive hidden elements of one token, sums the k BF16 expert rows
// in slot order in fp32, adds the (optionally gated) shared-expert row and
// rounds once to BF16.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float4 bf16x4(uint2 b) {
  return make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xffff0000u), __uint_as_float(b.y << 16),
                     __uint_as_float(b.y & 0xffff0000u));
}

__global__ void __launch_bounds__(kThreads)
combine_kernel(const zmoe_combine_args a) {
  const int t = blockIdx.y;
  const int h = (blockIdx.x * kThreads + threadIdx.x) * 4;
  if (h >= a.H) return;
  const int H = a.H, k = a.k;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.mode == ZMOE_ROUTE_SWITCH) {
    const int r = a.row_of[(size_t)t * k];
    const float w = a.topk_w[(size_t)t * k];
    const uint16_t* src = r >= 0 ? a.y + (size_t)r * H + h : a.x + (size_t)t * H + h;
    const float4 v = bf16x4(__ldg(reinterpret_cast<const uint2*>(src)));
    acc = make_float4(w * v.x, w * v.y, w * v.z, w * v.w);
  } else {
    for (int j = 0; j < k; ++j) {
      const int r = a.row_of[(size_t)t * k + j];
      if (r < 0) continue;
      const float w = a.topk_w[(size_t)t * k + j];
      const float4 v = bf16x4(__ldg(reinterpret_cast<const uint2*>(a.y + (size_t)r * H + h)));
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    if (a.y_shared) {
      const float g = a.shared_gate ? a.shared_gate[t] : 1.0f;
      const float4 v = bf16x4(__ldg(reinterpret_cast<const uint2*>(a.y_shared + (size_t)t * H + h)));
      acc.x = fmaf(g, v.x, acc.x);
      acc.y = fmaf(g, v.y, acc.y);
      acc.z = fmaf(g, v.z, acc.z);
      acc.w = fmaf(g, v.w, acc.w);
    }
  }
  uint2 o;
  o.x = (uint32_t)f32_to_bf16_bits(acc.x) | ((uint32_t)f32_to_bf16_bits(acc.y) << 16);
  o.y = (uint32_t)f32_to_bf16_bits(acc.z) | ((uint32_t)f32_to_bf16_bits(acc.w) << 16);
  *reinterpret_cast<uint2*>(a.out + (size_t)t * H + h) = o;
}

}  // namespace

zmoe_status launch_combine(const zmoe_combine_args* a, cudaStream_t stream) {
  ZMOE_CHECK_ARG(a && a->y && a->row_of && a->topk_w && a->out, "combine: null pointer");
  ZMOE_CHECK_ARG(a->H % 4 == 0, "combine: H must be a multiple of 4");
  ZMOE_CHECK_ARG(a->mode != ZMOE_ROUTE_SWITCH || a->x, "combine: Switch needs x for dropped tokens");
  if (a->T <= 0) return ZMOE_OK;
  dim3 grid((a->H / 4 + kThreads - 1) / kThreads, a->T);
  combine_kernel<<<grid, kThreads, 0, stream>>>(*a);
  return launch_status("combine_kernel");
}

}  // namespace zmoe
