// Permute (K3): per-expert counts, capacity drops, row assignment and the
// activation gather.
//
// Reference: ExpertExecutor.dispatch_local counts tokens per expert
// (experts/expert_executor.py:45-49) and ExpertDispatcher::GPUFetchFunc
// gathers them with a boolean mask, tokens ascending
// (csrc/dispatcher/expert_dispatcher.cpp:326-330).  The Switch capacity mask
// is the cumsum over the sequence axis of the transformers<4.47 Top1 router.
//
// Three small launches: (1) one CTA per expert ranks its tokens in token order
// with a block scan, drops those past the capacity of their sequence and writes
// the count; (2) one CTA per expert turns counts into offsets and writes
// row_of / token_of_row in the same order; (3) a grid-stride copy gathers the
// activation rows with 16-byte accesses.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kThreads = 256;

// Exclusive block scan of v (0/1 flags); returns the prefix, *total gets the sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += o;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (threadIdx.x < 32) {
    int s = threadIdx.x < kThreads / 32 ? warp_sums[threadIdx.x] : 0;
    int si = s;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, si, d);
      if ((int)threadIdx.x >= d) si += o;
    }
    if (threadIdx.x < kThreads / 32) warp_sums[threadIdx.x] = si - s;   // exclusive
    if (threadIdx.x == kThreads / 32 - 1) warp_sums[kThreads / 32] = si;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  *total = warp_sums[kThreads / 32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int slot_of(const int32_t* idx, int t, int k, int e) {
  for (int j = 0; j < k; ++j)
    if (idx[(size_t)t * k + j] == e) return j;
  return -1;
}

__global__ void __launch_bounds__(kThreads)
count_kernel(int32_t* __restrict__ topk_idx, int T, int k, int capacity, int seq_len,
             int32_t* __restrict__ counts) {
  __shared__ int warp_sums[kThreads / 32 + 1];
  const int e = blockIdx.x;
  const int row_len = capacity > 0 ? seq_len : T;
  int kept = 0;
  for (int r0 = 0; r0 < T; r0 += row_len) {
    const int r1 = min(T, r0 + row_len);
    int running = 0;
    for (int t0 = r0; t0 < r1; t0 += kThreads) {
      const int t = t0 + threadIdx.x;
      const int j = t < r1 ? slot_of(topk_idx, t, k, e) : -1;
      int total;
      const int rank = running + block_exclusive_scan(j >= 0 ? 1 : 0, warp_sums, &total);
      const bool drop = j >= 0 && capacity > 0 && rank >= capacity;
      if (drop) topk_idx[(size_t)t * k + j] = -1;
      kept += __syncthreads_count(j >= 0 && !drop);
      running += total;
    }
  }
  if (threadIdx.x == 0) counts[e] = kept;
}

__global__ void __launch_bounds__(kThreads)
scatter_kernel(const int32_t* __restrict__ topk_idx, int T, int k, int E,
               const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
               int32_t* __restrict__ row_of, int32_t* __restrict__ token_of_row) {
  __shared__ int warp_sums[kThreads / 32 + 1];
  __shared__ int base_s;
  const int e = blockIdx.x;
  if (threadIdx.x == 0) {
    int s = 0;
    for (int q = 0; q < e; ++q) s += counts[q];
    base_s = s;
    if (e == E - 1) {
      int acc = 0;
      for (int q = 0; q < E; ++q) { offsets[q] = acc; acc += counts[q]; }
      offsets[E] = acc;
    }
  }
  __syncthreads();
  const int base = base_s;
  int running = 0;
  for (int t0 = 0; t0 < T; t0 += kThreads) {
    const int t = t0 + threadIdx.x;
    const int j = t < T ? slot_of(topk_idx, t, k, e) : -1;
    int total;
    const int rank = running + block_exclusive_scan(j >= 0 ? 1 : 0, warp_sums, &total);
    if (j >= 0) {
      const int row = base + rank;
      row_of[(size_t)t * k + j] = row;
      token_of_row[row] = t;
    }
    running += total;
  }
}

__global__ void __launch_bounds__(kThreads)
gather_kernel(const uint16_t* __restrict__ x, int H, const int32_t* __restrict__ offsets, int E,
              const int32_t* __restrict__ token_of_row, uint16_t* __restrict__ xp, int max_rows) {
  const int rows = min(offsets[E], max_rows);
  const int vec = H / 8;
  const size_t total = (size_t)rows * vec;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int r = (int)(i / vec);
    const int c = (int)(i % vec);
    const int t = token_of_row[r];
    reinterpret_cast<uint4*>(xp + (size_t)r * H)[c] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H) + c);
  }
}

// dst[r] = src[index[r]], 16 bytes per thread and step.
__global__ void __launch_bounds__(kThreads)
gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ index, int rows, int vec,
                   uint4* __restrict__ dst) {
  const size_t total = (size_t)rows * vec;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const size_t r = i / vec;
    const int c = (int)(i % vec);
    dst[r * vec + c] = __ldg(src + (size_t)__ldg(index + r) * vec + c);
  }
}

}  // namespace

zmoe_status launch_permute(const zmoe_permute_args* a, cudaStream_t stream) {
  ZMOE_CHECK_ARG(a && a->topk_idx && a->counts && a->offsets && a->row_of && a->token_of_row,
                 "permute: null pointer");
  ZMOE_CHECK_ARG(a->E >= 1 && a->k >= 1, "permute: bad E/k");
  ZMOE_CHECK_ARG(a->capacity <= 0 || (a->seq_len > 0 && a->T % a->seq_len == 0),
                 "permute: T=%d must be a multiple of seq_len=%d when capacity is set", a->T, a->seq_len);
  ZMOE_CHECK_ARG(a->xp == nullptr || (a->x && a->H % 8 == 0 && (uintptr_t)a->x % 16 == 0 && (uintptr_t)a->xp % 16 == 0),
                 "permute: gather needs H %% 8 == 0 and 16-byte aligned x/xp");
  ZMOE_CUDA_RET(cudaMemsetAsync(a->row_of, 0xff, sizeof(int32_t) * (size_t)a->T * a->k, stream));
  if (a->T <= 0) {
    ZMOE_CUDA_RET(cudaMemsetAsync(a->counts, 0, sizeof(int32_t) * a->E, stream));
    ZMOE_CUDA_RET(cudaMemsetAsync(a->offsets, 0, sizeof(int32_t) * (a->E + 1), stream));
    return ZMOE_OK;
  }
  count_kernel<<<a->E, kThreads, 0, stream>>>(a->topk_idx, a->T, a->k, a->capacity, a->seq_len, a->counts);
  zmoe_status st = launch_status("count_kernel");
  if (st != ZMOE_OK) return st;
  scatter_kernel<<<a->E, kThreads, 0, stream>>>(a->topk_idx, a->T, a->k, a->E, a->counts, a->offsets,
                                                a->row_of, a->token_of_row);
  st = launch_status("scatter_kernel");
  if (st != ZMOE_OK || a->xp == nullptr) return st;
  const int max_rows = a->T * a->k;
  size_t blocks = ((size_t)max_rows * (a->H / 8) + kThreads - 1) / kThreads;
  if (blocks > (size_t)kNumSMs * 8) blocks = (size_t)kNumSMs * 8;
  if (blocks == 0) blocks = 1;
  gather_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(a->x, a->H, a->offsets, a->E, a->token_of_row,
                                                            a->xp, max_rows);
  return launch_status("gather_kernel");
}

zmoe_status launch_gather_rows(const void* src, const int32_t* index, int rows, int row_bytes, void* dst,
                               cudaStream_t stream) {
  ZMOE_CHECK_ARG(rows >= 0 && row_bytes > 0 && row_bytes % 16 == 0, "gather_rows: rows=%d, row_bytes=%d (multiple of 16)",
                 rows, row_bytes);
  if (rows == 0) return ZMOE_OK;
  ZMOE_CHECK_ARG(src && index && dst && (uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0,
                 "gather_rows: null or unaligned pointer");
  const int vec = row_bytes / 16;
  size_t blocks = ((size_t)rows * vec + kThreads - 1) / kThreads;
  if (blocks > (size_t)kNumSMs * 8) blocks = (size_t)kNumSMs * 8;
  gather_rows_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(static_cast<const uint4*>(src), index, rows, vec,
                                                                static_cast<uint4*>(dst));
  return launch_status("gather_rows_kernel");
}

}  // namespace zmoe
