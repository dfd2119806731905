// Router: logits, softmax, top-k (K2).
//
// Replaces Qwen2MoEBlock.__prepare_expert_route (customized/qwen.py:44-54),
// the DeepSeek greedy MoEGate (models/deepseek/modeling_deepseek.py:424-476)
// and the transformers<4.47 SwitchTransformersTop1Router probabilities/argmax.
//
// One CTA of 8 warps per token.  The token row sits in shared memory; warp w
// computes the logits of experts w, w+8, ... with lane l summing h = 256j + 8l + i
// (j outer, i inner) in fp32 and an xor-butterfly fold, an order the oracle
// reproduces exactly (products of two bf16 values are exact in fp32).  Warp 0
// then applies the bias and the mode's rounding, the softmax (exp_poly, strided
// lane sums, butterfly, IEEE divide) and k rounds of warp arg-max with ties to
// the lower index.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxE = 256;
constexpr int kMaxH = 8192;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float dot_row(const uint16_t* xs, const uint16_t* __restrict__ w, int H, int lane) {
  float acc = 0.0f;
  for (int j = 0; j < H / 256; ++j) {
    const int h = 256 * j + 8 * lane;
    const uint4 xv = *reinterpret_cast<const uint4*>(xs + h);
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + h));
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float x0 = __uint_as_float(xw[q] << 16), x1 = __uint_as_float(xw[q] & 0xffff0000u);
      const float w0 = __uint_as_float(ww[q] << 16), w1 = __uint_as_float(ww[q] & 0xffff0000u);
      acc = __fadd_rn(acc, __fmul_rn(x0, w0));
      acc = __fadd_rn(acc, __fmul_rn(x1, w1));
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, off));
  return acc;
}

// true when (va, ia) ranks before (vb, ib): larger value first, then lower index
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(kThreads)
router_kernel(const zmoe_router_args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);
  float* lg = reinterpret_cast<float*>(smem_raw + a.H * sizeof(uint16_t));  // [E + 1]
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, E = a.E;

  const uint4* xr = reinterpret_cast<const uint4*>(a.x + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += kThreads) reinterpret_cast<uint4*>(xs)[i] = __ldg(xr + i);
  __syncthreads();

  const int rows = E + (a.w_shared_gate ? 1 : 0);
  for (int e = warp; e < rows; e += kThreads / 32) {
    const uint16_t* w = e < E ? a.w + (size_t)e * H : a.w_shared_gate;
    const float v = dot_row(xs, w, H, lane);
    if (lane == 0) lg[e] = v;
  }
  __syncthreads();
  if (warp != 0) return;

  // ---- per-lane experts e = lane + 32 * j ----------------------------------
  constexpr int kPer = kMaxE / 32;
  float l[kPer], p[kPer];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    float v = -INFINITY;
    if (e < E) {
      v = lg[e];
      if (a.bias) v = __fadd_rn(v, a.bias[e]);
      if (a.mode == ZMOE_ROUTE_QWEN) v = round_bf16(v);
      if (a.logits) a.logits[(size_t)t * E + e] = v;
    }
    l[j] = v;
    m = fmaxf(m, v);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
  float part = 0.0f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < E ? exp_poly(__fsub_rn(l[j], m)) : 0.0f;
    if (j * 32 < E) part = __fadd_rn(part, p[j]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(kFull, part, off));
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      p[j] = __fdiv_rn(p[j], part);
      if (a.mode == ZMOE_ROUTE_SWITCH) p[j] = round_bf16(p[j]);
    } else {
      p[j] = -INFINITY;
    }
  }

  // ---- top-k --------------------------------------------------------------------
  float sel_v[8];
  int sel_i[8];
  const int k = a.k;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E && better(p[j], e, bv, bi)) { bv = p[j]; bi = e; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(kFull, bv, off);
      const int oi = __shfl_xor_sync(kFull, bi, off);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    sel_v[r] = bv;
    sel_i[r] = bi;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (lane + 32 * j == bi) p[j] = -INFINITY;       // remove from later rounds
  }
  if (lane == 0) {
    float s = 0.0f;
    if (a.norm_topk_prob && a.mode != ZMOE_ROUTE_SWITCH)
      for (int r = 0; r < k; ++r) s = __fadd_rn(s, sel_v[r]);
    for (int r = 0; r < k; ++r) {
      float w = sel_v[r];
      if (a.mode == ZMOE_ROUTE_QWEN) {
        if (a.norm_topk_prob) w = __fdiv_rn(w, s);
        w = round_bf16(w);
      } else if (a.mode == ZMOE_ROUTE_DEEPSEEK) {
        w = a.norm_topk_prob ? __fdiv_rn(w, __fadd_rn(s, 1e-20f)) : __fmul_rn(w, a.scaling);
      }
      a.topk_idx[(size_t)t * k + r] = sel_i[r];
      a.topk_w[(size_t)t * k + r] = w;
    }
    if (a.w_shared_gate && a.shared_gate) {
      const float g = round_bf16(lg[E]);
      a.shared_gate[t] = 1.0f / (1.0f + expf(-g));
    }
  }
}

}  // namespace

zmoe_status launch_router(const zmoe_router_args* a, cudaStream_t stream) {
  ZMOE_CHECK_ARG(a && a->x && a->w && a->topk_idx && a->topk_w, "router: null pointer");
  ZMOE_CHECK_ARG(a->H % 256 == 0 && a->H <= kMaxH, "router: H=%d must be a multiple of 256 and <= %d", a->H, kMaxH);
  ZMOE_CHECK_ARG(a->E >= 1 && a->E <= kMaxE, "router: E=%d outside [1, %d]", a->E, kMaxE);
  ZMOE_CHECK_ARG(a->k >= 1 && a->k <= 8 && a->k <= a->E, "router: k=%d outside [1, min(8, E)]", a->k);
  ZMOE_CHECK_ARG(a->mode >= 0 && a->mode <= 2, "router: bad mode %d", a->mode);
  ZMOE_CHECK_ARG(a->mode != ZMOE_ROUTE_SWITCH || a->k == 1, "router: Switch routing is top-1");
  ZMOE_CHECK_ARG((uintptr_t)a->x % 16 == 0 && (uintptr_t)a->w % 16 == 0, "router: x and w must be 16-byte aligned");
  if (a->T <= 0) return ZMOE_OK;
  const size_t smem = (size_t)a->H * 2 + (size_t)(a->E + 1) * 4;
  router_kernel<<<a->T, kThreads, smem, stream>>>(*a);
  return launch_status("router_kernel");
}

}  // namespace zmoe
