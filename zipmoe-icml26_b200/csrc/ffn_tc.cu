// Grouped expert FFN on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// Replaces DeepSeekMoEDenseActDense::forward / SwitchTransformersDenseActDense::forward
// (csrc/dispatcher/expert_module.cpp:39-50, :67-78), which the reference runs one
// expert at a time with three libtorch matmuls and a stream synchronisation
// around each expert (csrc/dispatcher/expert_dispatcher.cpp:354-427).
//
// Two persistent launches per layer:
//   up:   h[t, i] = bf16( silu(sum_k Wg[i,k] x[t,k]) * sum_k Wu[i,k] x[t,k] )   (or relu(Wi x))
//   down: y[t, j] = bf16( sum_i Wd[j,i] h[t,i] )
// Both are "swap-AB" GEMMs: the weight rows are the MMA M dimension (128 per
// tile), the group's tokens are the N dimension (up to 128 per tile), so a
// group with a handful of tokens still streams its weights at full width.
//
// CTA = 6 warps: warp 0 issues TMA (one lane), warp 1 allocates TMEM and issues
// tcgen05.mma (one lane), warps 2-5 run the epilogue from TMEM (warp w reads
// TMEM lanes 32*(w%4)..+31).  Operands land in shared memory through 2D tensor
// maps with 128-byte swizzle (K-major, 64 bf16 per row); a 4-stage (up) or
// 6-stage (down) mbarrier ring overlaps loads with MMAs.  Accumulators: fp32
// in TMEM, two of them, so the MMAs of a CTA's next unit run while the
// epilogue drains the last one (up: gate at columns 0..127 and up at 128..255
// of each 256-column accumulator; down: 128 columns each).  The 192 KB operand
// ring keeps one CTA per SM, so the 512 columns are always free.
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error code
// in zmoe's device error word (g_kernel_error, read by zmoe_kernel_error) and
// in the launch's own error word when the caller gave one, waits (bounded)
// for the loads it issued, releases its TMEM and returns.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace zmoe {

__device__ int32_t g_kernel_error = 0;

namespace tc {

constexpr int BM = 128;               // weight rows per tile (MMA M)
constexpr int BN = 128;               // tokens per tile of grouped launches (the narrow kernel's maximum)
constexpr int BNW = 256;              // tokens per tile at most in the wide kernel (max MMA N)
constexpr int BK = 64;                // bf16 per 128-byte swizzle row
constexpr int kTileBytes = BM * BK * 2;   // 16 KiB (A tile; B tile has the same size)
constexpr int kMaxMaps = 128;
constexpr int kMaxGroups = 128;
constexpr int kThreads = 192;
constexpr long long kWaitCycles = 4000000000LL;   // about 2 s at 1.9 GHz

// Error-path test hook (zmoe_debug_ffn_wait): the wait limit of the next
// launches, and whether their TMA producer issues nothing, so that the MMA
// warp's first wait runs out.  Host-side settings, copied into each launch.
long long g_wait_limit = kWaitCycles;
int g_drop_loads = 0;

struct __align__(64) Params {
  CUtensorMap amap[kMaxMaps];         // weight (A) maps: MODE 0 uses 2 per group
  CUtensorMap bmap;                   // activation (B) map over [rows_total, K]
  const int32_t* offsets;             // [G_all + 1] device, or nullptr: one group of rows_total
  void* out;                          // h or y (BF16), row-major [rows_total, n_out]
  int g_begin, g_count;               // groups of this launch (offset into offsets)
  int rows_total, K, n_out;           // n_out = weight rows of one matrix (I or H)
  int bn;                             // tokens per tile (multiple of 16, at most the kernel's BNT)
  int32_t* err;                       // caller's error word (device) or nullptr
  long long wait_limit;               // clock64 cycles a wait may take
  int drop_loads;                     // error-path test: the producer issues nothing
  uint8_t present[kMaxGroups];        // 0: group not in this launch (no weights)
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false on timeout (error recorded in the CTA, the device-wide
// word and the caller's word) or when another warp of the CTA already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* cta_err, int32_t* err_out,
                                          long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*(volatile int32_t*)cta_err) return false;
    if (clock64() - t0 > limit) {
      atomicCAS(cta_err, 0, 1);
      atomicCAS(&g_kernel_error, 0, 1);
      if (err_out) atomicCAS(err_out, 0, 1);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major operand tile in 128-byte-swizzled layout: rows of 128 bytes, 8-row
// atoms of 1024 bytes (stride-byte offset), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M = 128.
__device__ __forceinline__ uint32_t instr_desc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
// MODE 0: SwiGLU up (gate+up maps), 1: ReLU up, 2: down (BF16 out).  BNT: the
// largest token tile (the B region of a stage and the accumulator width); the
// launch's tile p.bn is at most BNT.
template <int MODE, int BNT>
__global__ void __launch_bounds__(kThreads, 1) ffn_tc_kernel(const __grid_constant__ Params p) {
  constexpr int NA = MODE == 0 ? 2 : 1;
  constexpr int kBTileBytes = BNT * BK * 2;
  constexpr int kStageBytes = NA * kTileBytes + kBTileBytes;
  constexpr int STAGES = (192 * 1024) / kStageBytes;     // 4 / 6 stages at BNT 128, 3 / 4 at 256
  constexpr uint32_t kAccCols = NA * BNT;                // TMEM columns of one accumulator
  constexpr uint32_t NACC = 2 * kAccCols <= 512 ? 2 : 1; // two accumulators (MMA and epilogue overlap) when they fit
  constexpr uint32_t kTmemCols = NACC * kAccCols;
  static_assert(STAGES >= 3 && STAGES <= 8, "operand ring depth");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;                // [2]
  uint64_t* tmem_empty = tmem_full + 2;               // [2]
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int32_t* cta_err = reinterpret_cast<int32_t*>(tmem_slot + 1);
  int32_t* prefix = cta_err + 1;              // [g_count + 1] tile prefix
  int32_t* ntiles = prefix + kMaxGroups + 1;  // [g_count] n tiles per group
  int32_t* row0 = ntiles + kMaxGroups;        // [g_count] first row of each group
  int32_t* rows = row0 + kMaxGroups;          // [g_count] rows of each group

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int MT = (p.n_out + BM - 1) / BM;     // partial tiles read zeros past the matrix edge
  const int KS = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);
    }
    mbar_init(drain, 1);
    *cta_err = 0;
    int acc = 0;
    for (int g = 0; g < p.g_count; ++g) {
      int r0 = 0, rn = p.rows_total;
      if (p.offsets) {
        r0 = p.offsets[p.g_begin + g];
        rn = p.offsets[p.g_begin + g + 1] - r0;
      }
      const int nt = (p.present[g] && rn > 0) ? (rn + p.bn - 1) / p.bn : 0;
      prefix[g] = acc;
      ntiles[g] = nt;
      row0[g] = r0;
      rows[g] = rn;
      acc += nt * MT;
    }
    prefix[p.g_count] = acc;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = prefix[p.g_count];

  auto unit_of = [&](int u, int& g, int& mt, int& nt) {
    int lo = 0, hi = p.g_count - 1;            // last g with prefix[g] <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    g = lo;
    const int local = u - prefix[g];
    mt = local / ntiles[g];
    nt = local % ntiles[g];
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed[8] = {0, 0, 0, 0, 0, 0, 0, 0};   // bit: stage armed in phase
      bool ok = true;
      for (int u = p.drop_loads ? total : (int)blockIdx.x; u < total && ok; u += gridDim.x) {
        int g, mt, nt;
        unit_of(u, g, mt, nt);
        const int arow = mt * BM;
        const int brow = row0[g] + nt * p.bn;
        const int m0 = MODE == 0 ? 2 * g : g;
        for (int ks = 0; ks < KS; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, cta_err, p.err, p.wait_limit)) { ok = false; break; }
          uint8_t* st = smem + stage * kStageBytes;
          mbar_expect_tx(&full[stage], NA * kTileBytes + p.bn * BK * 2);
          armed[stage] = phase + 1;
          tma_load_2d(st, &p.amap[m0], ks * BK, arow, &full[stage]);
          if (NA == 2) tma_load_2d(st + kTileBytes, &p.amap[m0 + 1], ks * BK, arow, &full[stage]);
          tma_load_2d(st + NA * kTileBytes, &p.bmap, ks * BK, brow, &full[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // drain: wait (bounded) for every load this lane issued
        for (int s = 0; s < STAGES; ++s)
          if (armed[s]) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], armed[s] - 1) && clock64() - t0 < p.wait_limit) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x, i = 0; u < total && ok; u += gridDim.x, ++i) {
        int g, mt, nt;
        unit_of(u, g, mt, nt);
        const int valid = min(p.bn, rows[g] - nt * p.bn);
        const int n = max(16, (valid + 15) & ~15);
        const uint32_t idesc = instr_desc(n);
        const int ab = (int)((uint32_t)i % NACC);       // accumulator of this unit
        const uint32_t acc_phase = ((uint32_t)i / NACC) & 1u;
        const uint32_t tacc = tmem + (uint32_t)ab * kAccCols;
        if (!mbar_wait(&tmem_empty[ab], acc_phase ^ 1u, cta_err, p.err, p.wait_limit)) break;
        tc_fence_after();
        for (int ks = 0; ks < KS; ++ks) {
          if (!mbar_wait(&full[stage], phase, cta_err, p.err, p.wait_limit)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint64_t da0 = smem_desc(sa);
          const uint64_t da1 = smem_desc(sa + kTileBytes);
          const uint64_t db = smem_desc(sa + NA * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t accf = (ks | kk) != 0;
            tc_mma(tacc, da0 + 2 * kk, db + 2 * kk, idesc, accf);
            if (NA == 2) tc_mma(tacc + BNT, da1 + 2 * kk, db + 2 * kk, idesc, accf);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit(&tmem_full[ab]);
      }
      if (!ok || *(volatile int32_t*)cta_err) {
        // error path: wait (bounded) until every MMA issued here has finished
        tc_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < p.wait_limit) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    for (int u = blockIdx.x, i = 0; u < total; u += gridDim.x, ++i) {
      int g, mt, nt;
      unit_of(u, g, mt, nt);
      const int valid = min(p.bn, rows[g] - nt * p.bn);
      const int n = max(16, (valid + 15) & ~15);
      const int ab = (int)((uint32_t)i % NACC);
      if (!mbar_wait(&tmem_full[ab], ((uint32_t)i / NACC) & 1u, cta_err, p.err, p.wait_limit)) break;
      tc_fence_after();
      const int feat = mt * BM + q * 32 + lane;   // output feature of this thread
      const size_t rbase = (size_t)(row0[g] + nt * p.bn);
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)ab * kAccCols;
      for (int c0 = 0; c0 < n; c0 += 16) {
        uint32_t a[16], b[16];
        tmem_ld16(taddr + c0, a);
        if (MODE == 0) tmem_ld16(taddr + BNT + c0, b);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = c0 + j;
          if (t >= valid || feat >= p.n_out) break;
          const size_t o = (rbase + t) * (size_t)p.n_out + feat;
          const float v = __uint_as_float(a[j]);
          if (MODE == 0) {
            static_cast<uint16_t*>(p.out)[o] = f32_to_bf16_bits(silu(v) * __uint_as_float(b[j]));
          } else if (MODE == 1) {
            static_cast<uint16_t*>(p.out)[o] = f32_to_bf16_bits(fmaxf(v, 0.0f));
          } else {
            static_cast<uint16_t*>(p.out)[o] = f32_to_bf16_bits(v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <int MODE, int BNT>
constexpr int smem_bytes() {
  constexpr int NA = MODE == 0 ? 2 : 1;
  constexpr int kStageBytes = NA * kTileBytes + BNT * BK * 2;
  constexpr int STAGES = (192 * 1024) / kStageBytes;
  return 1024 + STAGES * kStageBytes + 2 * STAGES * 8 + 40 + 8 + 4 * (4 * kMaxGroups + 2);
}

// Token tile of a launch with one dense group of R rows (the shared expert):
// the units (MT weight tiles x token tiles) should fill the SMs in whole
// waves.  A unit streams (NA * 128 + bn) * K * 2 bytes at about 100 GB/s per SM
// and runs 2 * NA * 128 * bn * K FLOP at about 10.7 TFLOP/s per SM; the tile
// with the least estimated waves x unit time wins.  Grouped launches keep BN.
inline int dense_tile(int MT, int R, int K, int NA, int sms) {
  int best = BN;
  double best_t = 1e30;
  for (int bn = 16; bn <= BNW; bn += 16) {
    const long long units = (long long)MT * ((R + bn - 1) / bn);
    const long long waves = (units + sms - 1) / sms;
    const double load = (double)(NA * BM + bn) * K * 2 / 100e9;
    const double mma = 2.0 * NA * BM * bn * (double)K / 10.7e12;
    const double t = (double)waves * (load > mma ? load : mma);
    if (t < best_t * 0.999) {
      best_t = t;
      best = bn;
    }
  }
  return best;
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// Encoded maps by (base, rows, cols, box rows).  A map holds only an address
// and a shape, so a cached one stays valid for any buffer at that address;
// the layer's slot, shared-expert and activation buffers keep their addresses,
// so after the first steps a launch encodes nothing on the host.
struct MapKey {
  uintptr_t base;
  uint64_t rows, cols;
  uint32_t box;
  bool operator==(const MapKey& o) const { return base == o.base && rows == o.rows && cols == o.cols && box == o.box; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.base * 0x9E3779B97F4A7C15ull;
    h ^= (k.rows + 0x632BE59BD9B4E019ull) + (h << 6) + (h >> 2);
    h ^= (k.cols * 31 + k.box + 0x8CB92BA72F3D8DD7ull) + (h << 6) + (h >> 2);
    return (size_t)h;
  }
};

zmoe_status encode_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

// 2D bf16 map over a row-major [rows, cols] matrix; box = BK columns x box_rows rows.
zmoe_status make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, box_rows};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *m = it->second;
    return ZMOE_OK;
  }
  zmoe_status st = encode_map(m, base, rows, cols, box_rows);
  if (st != ZMOE_OK) return st;
  if (cache.size() >= 8192) cache.clear();         // bounded: callers with ever-new buffers re-encode
  cache.emplace(key, *m);
  return ZMOE_OK;
}

zmoe_status encode_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is not available");
    return ZMOE_ECUDA;
  }
  ZMOE_CHECK_ARG(((uintptr_t)base & 15) == 0, "tensor map base %p is not 16-byte aligned", base);
  ZMOE_CHECK_ARG((cols * 2) % 16 == 0, "row pitch %llu bytes is not a multiple of 16", (unsigned long long)cols * 2);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for %llux%llu at %p", (int)r, (unsigned long long)rows,
              (unsigned long long)cols, base);
    return ZMOE_ECUDA;
  }
  return ZMOE_OK;
}

template <int MODE>
zmoe_status launch_mode(const zmoe_ffn_args* a, const uint16_t* act, int K, int n_out, void* out,
                        cudaStream_t stream, int32_t* err) {
  const int per = MODE == 0 ? 2 : 1;
  const int gmax = kMaxMaps / per < kMaxGroups ? kMaxMaps / per : kMaxGroups;
  static Params p;                            // 17 KB: too large for the stack frame of a host thread loop
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int dev = 0, sms = kNumSMs;
  ZMOE_CUDA_RET(cudaGetDevice(&dev));
  ZMOE_CUDA_RET(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int bn = a->offsets ? BN : dense_tile((n_out + BM - 1) / BM, a->rows_total, K, per, sms);
  const bool wide = bn > BN;
  const int smem = wide ? smem_bytes<MODE, BNW>() : smem_bytes<MODE, BN>();
  static uint64_t attr_set[2] = {0, 0};              // per kernel variant: devices whose attribute is set
  const uint64_t dbit = 1ull << (dev & 63);
  if (!(attr_set[wide] & dbit)) {
    if (wide)
      ZMOE_CUDA_RET(cudaFuncSetAttribute(ffn_tc_kernel<MODE, BNW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    else
      ZMOE_CUDA_RET(cudaFuncSetAttribute(ffn_tc_kernel<MODE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set[wide] |= dbit;
  }
  for (int g0 = 0; g0 < a->G; g0 += gmax) {
    const int gc = a->G - g0 < gmax ? a->G - g0 : gmax;
    memset(&p, 0, sizeof(p));
    int any = 0;
    for (int g = 0; g < gc; ++g) {
      const uint16_t* const* wg = a->w + 3 * (size_t)(g0 + g);
      const uint16_t* m0 = MODE == 2 ? wg[2] : wg[0];
      const uint16_t* m1 = MODE == 0 ? wg[1] : nullptr;
      if (!m0 || (MODE == 0 && !m1)) continue;
      zmoe_status st = make_map(&p.amap[per * g], m0, (uint64_t)n_out, (uint64_t)K, BM);
      if (st == ZMOE_OK && MODE == 0) st = make_map(&p.amap[per * g + 1], m1, (uint64_t)n_out, (uint64_t)K, BM);
      if (st != ZMOE_OK) return st;
      p.present[g] = 1;
      any = 1;
    }
    if (!any) continue;
    zmoe_status st = make_map(&p.bmap, act, (uint64_t)a->rows_total, (uint64_t)K, (uint32_t)bn);
    if (st != ZMOE_OK) return st;
    p.offsets = a->offsets;
    p.out = out;
    p.g_begin = g0;
    p.g_count = gc;
    p.rows_total = a->rows_total;
    p.K = K;
    p.n_out = n_out;
    p.bn = bn;
    p.err = err;
    p.wait_limit = g_wait_limit;
    p.drop_loads = g_drop_loads;
    if (wide) ffn_tc_kernel<MODE, BNW><<<sms, kThreads, smem, stream>>>(p);
    else ffn_tc_kernel<MODE, BN><<<sms, kThreads, smem, stream>>>(p);
    st = launch_status("ffn_tc_kernel");
    if (st != ZMOE_OK) return st;
  }
  return ZMOE_OK;
}

}  // namespace tc

// a->w is a host array of G*3 device pointers.  err: device error word that
// a timed-out wait sets to 1 (nullptr: only the device-wide word is set).
zmoe_status launch_expert_ffn(const zmoe_ffn_args* a, cudaStream_t stream, int32_t* err) {
  ZMOE_CHECK_ARG(a && a->x && a->w && a->h && a->y, "expert_ffn: null pointer");
  ZMOE_CHECK_ARG(a->G >= 1, "expert_ffn: G must be >= 1");
  ZMOE_CHECK_ARG(a->kind == 0 || a->kind == 1, "expert_ffn: kind must be 0 (SwiGLU) or 1 (ReLU)");
  ZMOE_CHECK_ARG(a->H > 0 && a->H % 8 == 0 && a->I > 0 && a->I % 8 == 0,
                 "expert_ffn: H=%d and I=%d must be positive multiples of 8", a->H, a->I);
  ZMOE_CHECK_ARG(a->offsets || a->G == 1, "expert_ffn: offsets required for G > 1");
  // A group takes part with all of its matrices or with none: the down pass
  // must never read an intermediate that the up pass did not write.
  for (int g = 0; g < a->G; ++g) {
    const uint16_t* const* w = a->w + 3 * (size_t)g;
    const bool up_set = w[0] && (a->kind == 1 || w[1]);
    const bool none = !w[0] && !w[1] && !w[2];
    ZMOE_CHECK_ARG(none || (up_set && w[2]),
                   "expert_ffn: group %d has only some of its weight pointers set (w0=%p w1=%p w2=%p)", g,
                   (const void*)w[0], (const void*)w[1], (const void*)w[2]);
  }
  if (a->rows_total <= 0) return ZMOE_OK;
  zmoe_status st = a->kind == 0 ? tc::launch_mode<0>(a, a->x, a->H, a->I, a->h, stream, err)
                                : tc::launch_mode<1>(a, a->x, a->H, a->I, a->h, stream, err);
  if (st != ZMOE_OK) return st;
  return tc::launch_mode<2>(a, a->h, a->I, a->H, a->y, stream, err);
}

zmoe_status read_kernel_error(int32_t* out, int reset) {
  ZMOE_CUDA_RET(cudaMemcpyFromSymbol(out, g_kernel_error, sizeof(int32_t)));
  if (reset) {
    const int32_t z = 0;
    ZMOE_CUDA_RET(cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(int32_t)));
  }
  return ZMOE_OK;
}

void set_ffn_wait(long long cycles, int drop_loads) {
  tc::g_wait_limit = cycles > 0 ? cycles : tc::kWaitCycles;
  tc::g_drop_loads = drop_loads != 0;
}

}  // namespace zmoe
