// Router: logits, softmax, top-k (K2).
//
// Replaces Qwen2MoEBlock.__prepare_expert_route (customized/qwen.py:44-54),
// the DeepSeek greedy MoEGate (models/deepseek/modeling_deepseek.py:424-476)
// and the transformers<4.47 SwitchTransformersTop1Router probabilities/argmax.
//
// One CTA of 16 warps per 4 tokens.  The token rows sit in shared memory (fp32);
// warp w computes the logits of experts w, w+16, ... for the 4 tokens (each
// weight load serves all 4) with lane l summing h = 256j + 8l + i (j outer, i
// inner) in fp32 by fused multiply-adds and an xor-butterfly fold, an order the
// oracle reproduces exactly (products of two bf16 values are exact in fp32, so
// fused and unfused multiply-add agree).  Warp w < 4 then
// applies, for token w, the bias and the mode's rounding, the softmax
// (exp_poly, strided lane sums, butterfly, IEEE divide) and k rounds of warp
// arg-max with ties to the lower index.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kTok = 4;                                // tokens per CTA
static_assert(kTok <= kWarps, "warp w finishes token w of the CTA");
constexpr int kMaxE = 256;
constexpr int kMaxH = 8192;
constexpr unsigned kFull = 0xffffffffu;

// The token rows are kept in fp32 in two planes: element h of a row sits in
// plane (h % 8) / 4 at (h / 8) * 4 + h % 4, so lane l's 8 elements of block j
// are one 16-byte load from each plane, conflict-free across the warp.
__device__ __forceinline__ int plane_idx(int h) { return (h >> 3) * 4 + (h & 3); }

// Adds blocks j0 .. j0 + n - 1 of one weight row (wv, this lane's 8 bf16 of
// each) to the kTok accumulators, in the fixed order per token (j outer, i
// inner).  A block's weights are unpacked once for all tokens.
template <int kTok>
__device__ __forceinline__ void dot_add(float (&acc)[kTok], const float* xs, int H, int j0, int lane,
                                        const uint4 (&wv)[8], int n) {
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) {
    if (jj >= n) break;
    const uint32_t ww[4] = {wv[jj].x, wv[jj].y, wv[jj].z, wv[jj].w};
    float wf[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      wf[2 * q] = __uint_as_float(ww[q] << 16);
      wf[2 * q + 1] = __uint_as_float(ww[q] & 0xffff0000u);
    }
    const int pi = (32 * (j0 + jj) + lane) * 4;        // plane index of h = 256(j0 + jj) + 8 lane
#pragma unroll
    for (int tk = 0; tk < kTok; ++tk) {
      const float* xr = xs + (size_t)tk * H;           // planes of token tk: [0, H/2) and [H/2, H)
      const float4 lo = *reinterpret_cast<const float4*>(xr + pi);
      const float4 hi = *reinterpret_cast<const float4*>(xr + H / 2 + pi);
      const float xf[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      // the product of two bf16 values is exact in fp32 (when it is not
      // subnormal), so the fused multiply-add rounds exactly as acc + (x * w)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[tk] = __fmaf_rn(xf[i], wf[i], acc[tk]);
    }
  }
}

// Loads h-blocks j0 .. j0 + n - 1 (n <= 8) of weight row w for lane l.
__device__ __forceinline__ void load_blocks(uint4 (&wv)[8], const uint16_t* __restrict__ w, int j0, int n, int lane) {
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) {
    if (jj >= n) break;
    wv[jj] = __ldg(reinterpret_cast<const uint4*>(w + 256 * (j0 + jj) + 8 * lane));
  }
}

// true when (va, ia) ranks before (vb, ib): larger value first, then lower index
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(kThreads)
router_kernel(const zmoe_router_args a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int H = a.H, E = a.E;
  float* xs = reinterpret_cast<float*>(smem_raw);                                  // [kTok][H], two planes each
  float* lgs = xs + (size_t)kTok * H;                                              // [kTok][E + 1]
  const int t0 = blockIdx.x * kTok;
  const int nt = a.T - t0 < kTok ? a.T - t0 : kTok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint4* xr = reinterpret_cast<const uint4*>(a.x + (size_t)t0 * H);   // the CTA's rows are contiguous
  for (int i = threadIdx.x; i < kTok * H / 8; i += kThreads) {
    const int tk = i / (H / 8), m = i % (H / 8);       // 8 elements h = 8m .. 8m + 7 of token tk
    uint4 v = make_uint4(0, 0, 0, 0);
    if (tk < nt) v = __ldg(xr + i);
    float* xp = xs + (size_t)tk * H + plane_idx(8 * m);
    *reinterpret_cast<float4*>(xp) = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                                                 __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
    *reinterpret_cast<float4*>(xp + H / 2) =
        make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u), __uint_as_float(v.w << 16),
                    __uint_as_float(v.w & 0xffff0000u));
  }
  __syncthreads();

  // warp w: rows w, w + kWarps, ..., each in chunks of 8 h-blocks; the next
  // chunk's weight loads are in flight while the current one is summed for
  // the CTA's tokens (one independent accumulator per token)
  const int rows = E + (a.w_shared_gate ? 1 : 0);
  auto row_ptr = [&](int e) { return e < E ? a.w + (size_t)e * H : a.w_shared_gate; };
  const int nj = H / 256, nch = (nj + 7) / 8;
  const int my_rows = warp < rows ? (rows - warp + kWarps - 1) / kWarps : 0;
  const int items = my_rows * nch;
  uint4 cur[8], nxt[8];
  if (items > 0) load_blocks(cur, row_ptr(warp), 0, nj < 8 ? nj : 8, lane);
  float acc[kTok];
  for (int i = 0; i < items; ++i) {
    const int e = warp + kWarps * (i / nch), c = i % nch;
    const int j0 = 8 * c, n = nj - j0 < 8 ? nj - j0 : 8;
    if (i + 1 < items) {
      const int e1 = warp + kWarps * ((i + 1) / nch), c1 = (i + 1) % nch;
      load_blocks(nxt, row_ptr(e1), 8 * c1, nj - 8 * c1 < 8 ? nj - 8 * c1 : 8, lane);
    }
    if (c == 0) {
#pragma unroll
      for (int tk = 0; tk < kTok; ++tk) acc[tk] = 0.0f;
    }
    dot_add<kTok>(acc, xs, H, j0, lane, cur, n);
    if (c == nch - 1) {
#pragma unroll
      for (int tk = 0; tk < kTok; ++tk) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc[tk] = __fadd_rn(acc[tk], __shfl_xor_sync(kFull, acc[tk], off));
      }
      if (lane == 0) {
#pragma unroll
        for (int tk = 0; tk < kTok; ++tk) lgs[tk * (E + 1) + e] = acc[tk];
      }
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) cur[jj] = nxt[jj];
  }
  __syncthreads();
  if (warp >= nt) return;                              // warp w finishes token t0 + w
  const int t = t0 + warp;
  const float* lg = lgs + warp * (E + 1);

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
  const size_t smem = (size_t)kTok * a->H * 4 + (size_t)kTok * (a->E + 1) * 4;
  if (smem > 48 * 1024) {                              // the largest size set so far, per device
    static int set_bytes[64] = {};
    int dev = 0;
    ZMOE_CUDA_RET(cudaGetDevice(&dev));
    if ((int)smem > set_bytes[dev & 63]) {
      ZMOE_CUDA_RET(cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      set_bytes[dev & 63] = (int)smem;
    }
  }
  router_kernel<<<(a->T + kTok - 1) / kTok, kThreads, smem, stream>>>(*a);
  return launch_status("router_kernel");
}

}  // namespace zmoe
