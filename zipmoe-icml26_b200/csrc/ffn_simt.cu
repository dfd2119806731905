// Grouped expert FFN, CUDA-core version (first correct path).
//
// Computes what DeepSeekMoEDenseActDense::forward / SwitchTransformersDenseActDense
// ::forward do (csrc/dispatcher/expert_module.cpp:39-50, :67-78) for all
// experts of a layer in two launches: gate/up (+SwiGLU or ReLU) into the BF16
// intermediate h, then down into fp32 y.  fp32 accumulation; h rounded once.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kBM = 32, kBN = 64, kBK = 32, kThreads = 256;

template <int MODE>  // 0: SwiGLU gate/up -> h ; 1: ReLU wi -> h ; 2: down -> y
__global__ void __launch_bounds__(kThreads)
ffn_simt_kernel(const uint16_t* __restrict__ A, const uint16_t* const* __restrict__ w,
                const int32_t* __restrict__ offsets, int rows_total, int K, int N,
                uint16_t* __restrict__ h, float* __restrict__ y) {
  __shared__ float As[kBM][kBK + 1];
  __shared__ float Bs[kBN][kBK + 1];
  __shared__ float Bu[MODE == 0 ? kBN : 1][kBK + 1];
  const int g = blockIdx.z;
  const int r0 = offsets ? offsets[g] : 0;
  const int r1 = offsets ? offsets[g + 1] : rows_total;
  const int row_base = r0 + blockIdx.y * kBM;
  if (row_base >= r1) return;
  const int col_base = blockIdx.x * kBN;
  const uint16_t* W0 = MODE == 2 ? w[3 * g + 2] : w[3 * g];
  const uint16_t* W1 = MODE == 0 ? w[3 * g + 1] : nullptr;
  if (W0 == nullptr || (MODE == 0 && W1 == nullptr)) return;   // group not in this launch
  const int tr = threadIdx.x / 16, tc = threadIdx.x % 16;
  float acc[2][4] = {}, accu[2][4] = {};
  for (int k0 = 0; k0 < K; k0 += kBK) {
    for (int i = threadIdx.x; i < kBM * kBK; i += kThreads) {
      const int rr = i / kBK, kk = i % kBK;
      const int r = row_base + rr, kx = k0 + kk;
      As[rr][kk] = (r < r1 && kx < K) ? bf16_bits_to_f32(A[(size_t)r * K + kx]) : 0.f;
    }
    for (int i = threadIdx.x; i < kBN * kBK; i += kThreads) {
      const int cc = i / kBK, kk = i % kBK;
      const int c = col_base + cc, kx = k0 + kk;
      const bool ok = c < N && kx < K;
      Bs[cc][kk] = ok ? bf16_bits_to_f32(W0[(size_t)c * K + kx]) : 0.f;
      if (MODE == 0) Bu[cc][kk] = ok ? bf16_bits_to_f32(W1[(size_t)c * K + kx]) : 0.f;
    }
    __syncthreads();
    for (int kk = 0; kk < kBK; ++kk) {
      const float a0 = As[tr * 2][kk], a1 = As[tr * 2 + 1][kk];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = Bs[tc * 4 + q][kk];
        acc[0][q] = fmaf(a0, b, acc[0][q]);
        acc[1][q] = fmaf(a1, b, acc[1][q]);
        if (MODE == 0) {
          const float u = Bu[tc * 4 + q][kk];
          accu[0][q] = fmaf(a0, u, accu[0][q]);
          accu[1][q] = fmaf(a1, u, accu[1][q]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = row_base + tr * 2 + i;
    if (r >= r1) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = col_base + tc * 4 + q;
      if (c >= N) continue;
      if (MODE == 0) {
        const float gv = acc[i][q];
        h[(size_t)r * N + c] = f32_to_bf16_bits(gv / (1.0f + expf(-gv)) * accu[i][q]);
      } else if (MODE == 1) {
        h[(size_t)r * N + c] = f32_to_bf16_bits(fmaxf(acc[i][q], 0.f));
      } else {
        y[(size_t)r * N + c] = acc[i][q];
      }
    }
  }
}

}  // namespace

zmoe_status launch_expert_ffn(const zmoe_ffn_args* a, cudaStream_t stream) {
  ZMOE_CHECK_ARG(a && a->x && a->w && a->h && a->y, "expert_ffn: null pointer");
  ZMOE_CHECK_ARG(a->G >= 1 && a->H > 0 && a->I > 0, "expert_ffn: bad sizes");
  ZMOE_CHECK_ARG(a->kind == 0 || a->kind == 1, "expert_ffn: kind must be 0 (SwiGLU) or 1 (ReLU)");
  if (a->rows_total <= 0) return ZMOE_OK;
  dim3 g1((a->I + kBN - 1) / kBN, (a->rows_total + kBM - 1) / kBM, a->G);
  if (a->kind == 0)
    ffn_simt_kernel<0><<<g1, kThreads, 0, stream>>>(a->x, a->w, a->offsets, a->rows_total, a->H, a->I, a->h, nullptr);
  else
    ffn_simt_kernel<1><<<g1, kThreads, 0, stream>>>(a->x, a->w, a->offsets, a->rows_total, a->H, a->I, a->h, nullptr);
  zmoe_status st = launch_status("ffn_simt up");
  if (st != ZMOE_OK) return st;
  dim3 g2((a->H + kBN - 1) / kBN, (a->rows_total + kBM - 1) / kBM, a->G);
  ffn_simt_kernel<2><<<g2, kThreads, 0, stream>>>(a->h, a->w, a->offsets, a->rows_total, a->I, a->H, nullptr, a->y);
  return launch_status("ffn_simt down");
}

}  // namespace zmoe
