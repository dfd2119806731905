// Fused LZ4-block decode + plane recombine (sm_100a).
//
// Reference path replaced: per exponent chunk, LZ4_decompress_safe_partial
// on a CPU worker (csrc/tensor_engine/compressors.cpp:195-211, driven by
// tensor_engine.cpp:421-474), a memcpy into a pinned dock, then the recombine
// kernel (csrc/kernels/tensor_recover.cu:12-43) reading both planes over
// zero-copy host memory.
//
// One CTA of 16 warps owns one LZ4 block.  A segment index built when the
// block is loaded (zmoe_lz4_build_index: the first sequence at or after every
// multiple of seg_bytes of output) lets warp w decode segments w, w+16, ...
// concurrently.  Inside a segment a warp walks batches of up to 32 sequences:
//
//  1. The compressed bytes from the current token are staged in shared memory
//     with aligned 32-bit loads; each lane computes, for 8 positions, where the
//     next token would start if one started there.  Pointer doubling over that
//     table gives lane l the start of sequence l in 5 shared-memory lookups.
//  2. Each lane decodes its sequence header; a warp scan gives output offsets;
//     an owner table maps every output byte of the batch to its sequence.
//  3. A match whose source lies in an earlier segment waits (bounded spin)
//     until the warp owning that segment has published a frontier past the
//     source; the warp owning the lowest unfinished segment never waits, so
//     the CTA always makes progress.
//  4. Output bytes are spread over the lanes by position (coalesced BF16
//     stores and sign+mantissa loads).  A literal comes from the staged
//     window; a match byte k of a copy with offset o reads position
//     (start - o + k mod o), which resolves overlapping copies directly.
//     The rare byte whose source is produced in the same batch is written in
//     a later round once its source is final.
//  5. Every exponent byte is merged with its sign+mantissa byte and stored as
//     BF16 in the destination slot; match sources are read back from the slot
//     through L2 (exponent = bits 7..14).
//
// Errors (bad offsets, lengths past the block, a block ending short of
// out_size, a wait that exceeds its bound) set the chunk's status word; the
// kernel never traps.  Output past out_size is clipped (the
// targetOutputSize = out_size behaviour of LZ4_decompress_safe_partial).
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kWarps = 16;
constexpr uint32_t kWin = 256;          // compressed bytes staged per batch
constexpr int kLevels = 5;              // jumps of 1, 2, 4, 8, 16 tokens
constexpr uint32_t kBatchMax = 1024;    // output bytes of one batch (owner table)
constexpr uint32_t kSpinLimit = 1u << 21;
constexpr unsigned kFull = 0xffffffffu;
constexpr int32_t kTimeout = 5;         // status: a dependency wait ran out

struct WarpSmem {
  uint32_t winw[kWin / 4 + 2];          // staged bytes, word aligned at the source
  uint16_t jump[kLevels][kWin];
  uint8_t owner[kBatchMax];
  uint32_t seq_ostart[32], seq_ms[32], seq_lit[32], seq_off[32];
  uint32_t pend[kBatchMax / 32];
};

struct CtaSmem {
  WarpSmem w[kWarps];
  uint32_t frontier[kWarps];            // output position final in the warp's current segment
  int32_t err;
};

__device__ __forceinline__ uint32_t vload(const volatile uint32_t* p) { return *p; }

// Start of the token after a token at window position i, or kWin when the
// chain cannot continue inside the staged bytes.
__device__ __forceinline__ uint32_t next_token(const uint8_t* win, uint32_t i, uint32_t avail, uint32_t rem) {
  if (i >= avail) return kWin;
  const uint32_t tok = win[i];
  uint32_t j = i + 1;
  uint32_t ll = tok >> 4;
  if (ll == 15) {
    uint32_t b;
    do {
      if (j >= avail) return kWin;
      b = win[j++];
      ll += b;
    } while (b == 255);
  }
  j += ll;
  if (j >= rem) return kWin;            // literals reach the block end: last sequence
  if (j + 2 > avail) return kWin;
  j += 2;
  if ((tok & 15) == 15) {
    uint32_t b;
    do {
      if (j >= avail) return kWin;
      b = win[j++];
    } while (b == 255);
  }
  return j < kWin ? j : kWin;
}

__device__ __forceinline__ uint32_t exp_of(const uint16_t* dst, uint32_t pos) {
  return ((uint32_t)__ldcg(dst + pos) >> 7) & 0xFFu;
}

struct Chunk {
  const uint8_t* src;
  const uint8_t* sm;
  uint16_t* dst;
  const uint32_t* index;
  uint32_t src_size, out_size, n_seg, seg_bytes;

  __device__ uint32_t seg_out(uint32_t j) const {  // output start of segment j
    return j >= n_seg ? out_size : min(__ldg(index + 2 * j + 1), out_size);
  }
  __device__ uint32_t seg_in(uint32_t j) const { return __ldg(index + 2 * j); }
  // segment holding output position q
  __device__ uint32_t seg_of(uint32_t q) const {
    uint32_t j = min(q / seg_bytes, n_seg - 1);
    while (j > 0 && seg_out(j) > q) --j;
    return j;
  }
};

// Wait until every byte of [a, b) (all before the caller's segment) is final.
__device__ bool wait_final(CtaSmem& S, const Chunk& c, uint32_t a, uint32_t b) {
  if (a >= b) return true;
  uint32_t j = c.seg_of(a);
  const uint32_t jb = c.seg_of(b - 1);
  for (; j <= jb; ++j) {
    const uint32_t need = min(b, c.seg_out(j + 1));
    const volatile uint32_t* f = &S.frontier[j % kWarps];
    uint32_t spins = 0;
    while (vload(f) < need) {
      if (*(volatile int32_t*)&S.err) return false;
      if (++spins > kSpinLimit) {
        atomicCAS(&S.err, 0, kTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  __threadfence_block();
  return true;
}

__device__ __forceinline__ void set_err(CtaSmem& S, int32_t code) { atomicCAS(&S.err, 0, code); }

__device__ __forceinline__ bool cta_failed(CtaSmem& S) { return *(volatile int32_t*)&S.err != 0; }

// Decode one segment [out_lo, out_hi) starting at token position in_lo.
__device__ void decode_segment(CtaSmem& S, WarpSmem& W, const Chunk& c, uint32_t in_lo, uint32_t out_lo,
                               uint32_t out_hi, uint32_t lane, int warp) {
  const uint8_t* win8 = reinterpret_cast<const uint8_t*>(W.winw);
  uint32_t ip = in_lo, op = out_lo;
  while (op < out_hi) {
    if (cta_failed(S)) return;
    if (ip >= c.src_size) { set_err(S, ZMOE_CHUNK_INPUT_OVERRUN); return; }
    // ---- stage compressed bytes [ip, ip + kWin) ---------------------------------
    const uint32_t rem = c.src_size - ip;
    const uint32_t avail = rem < kWin ? rem : kWin;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(c.src) + ip;
    const uint32_t shift = (uint32_t)(addr & 3);
    const uint32_t* wbase = reinterpret_cast<const uint32_t*>(addr - shift);
    const uintptr_t beg_addr = reinterpret_cast<uintptr_t>(c.src);
    const uintptr_t end_addr = beg_addr + c.src_size;
    for (uint32_t q = lane; q < kWin / 4 + 2; q += 32) {
      const uintptr_t wa = addr - shift + 4 * q;
      uint32_t v = 0;
      if (wa >= beg_addr && wa + 4 <= end_addr) {
        v = __ldg(wbase + q);
      } else {
        for (uint32_t b = 0; b < 4; ++b)
          if (wa + b >= beg_addr && wa + b < end_addr)
            v |= (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(wa + b)) << (8 * b);
      }
      W.winw[q] = v;
    }
    __syncwarp();
    const uint8_t* win = win8 + shift;
#pragma unroll
    for (uint32_t q = 0; q < kWin / 32; ++q) {
      const uint32_t i = lane * (kWin / 32) + q;
      W.jump[0][i] = (uint16_t)next_token(win, i, avail, rem);
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k + 1 < kLevels; ++k) {
#pragma unroll
      for (uint32_t q = 0; q < kWin / 32; ++q) {
        const uint32_t i = lane * (kWin / 32) + q;
        const uint32_t v = W.jump[k][i];
        W.jump[k + 1][i] = v < kWin ? W.jump[k][v] : (uint16_t)kWin;
      }
      __syncwarp();
    }
    uint32_t p = 0;
#pragma unroll
    for (int k = 0; k < kLevels; ++k)
      if ((lane >> k) & 1) p = p < kWin ? W.jump[k][p] : kWin;
    bool valid = p < avail;

    // ---- sequence header of this lane ----------------------------------------------
    auto byte_at = [&](uint32_t pos) -> uint32_t {
      const uint32_t rel = pos - ip;
      return rel < avail ? (uint32_t)win[rel] : (uint32_t)__ldg(c.src + pos);
    };
    uint32_t ll = 0, ml = 0, off = 0, lit_pos = 0, seq_end = 0;
    int lerr = 0;
    if (valid) {
      const uint32_t tok = win[p];
      uint32_t q = ip + p + 1;
      ll = tok >> 4;
      if (ll == 15) {
        uint32_t b;
        do {
          if (q >= c.src_size) { lerr = ZMOE_CHUNK_INPUT_OVERRUN; break; }
          b = byte_at(q++);
          ll += b;
        } while (b == 255 && ll < (1u << 30));
      }
      lit_pos = q;
      if (!lerr) {
        if ((uint64_t)q + ll > c.src_size) {
          lerr = ZMOE_CHUNK_INPUT_OVERRUN;
        } else {
          q += ll;
          if (q != c.src_size) {
            if (q + 2 > c.src_size) {
              lerr = ZMOE_CHUNK_INPUT_OVERRUN;
            } else {
              off = byte_at(q) | (byte_at(q + 1) << 8);
              q += 2;
              ml = tok & 15;
              if (ml == 15) {
                uint32_t b;
                do {
                  if (q >= c.src_size) { lerr = ZMOE_CHUNK_INPUT_OVERRUN; break; }
                  b = byte_at(q++);
                  ml += b;
                } while (b == 255 && ml < (1u << 30));
              }
              ml += 4;
            }
          }
        }
      }
      seq_end = q;
    }
    // output offsets
    const uint64_t len = valid ? (uint64_t)ll + ml : 0;
    uint64_t incl = len;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint64_t v = __shfl_up_sync(kFull, incl, d);
      if (lane >= (uint32_t)d) incl += v;
    }
    const uint64_t ostart = (uint64_t)op + incl - len;
    valid = valid && ostart < out_hi;                         // sequences of this segment only
    const uint64_t oend = min(ostart + len, (uint64_t)out_hi); // clip (partial decode target)
    // a batch holds the leading lanes whose output stays inside kBatchMax
    const unsigned fit = __ballot_sync(kFull, valid && oend - op <= kBatchMax);
    const unsigned vmask = __ballot_sync(kFull, valid);
    int cnt = __popc(vmask);                                   // valid lanes are a prefix
    int nb = __ffs(~fit) - 1;                                  // leading fitting lanes
    if (fit == kFull) nb = 32;
    nb = min(nb, cnt);
    const bool long_mode = nb == 0;                            // lane 0 alone exceeds kBatchMax
    const int used = long_mode ? 1 : nb;
    const bool mine = (int)lane < used;
    // errors of the lanes that take part
    const uint64_t ms = ostart + ll;
    if (mine && !lerr && ml > 0 && ms < oend && (off == 0 || off > ms)) lerr = ZMOE_CHUNK_BAD_OFFSET;
    const unsigned emask = __ballot_sync(kFull, mine && lerr != 0);
    if (emask) {
      set_err(S, __shfl_sync(kFull, lerr, __ffs(emask) - 1));
      return;
    }
    const uint32_t bs = op;
    const uint32_t be = (uint32_t)__shfl_sync(kFull, oend, used - 1);
    const uint32_t seg_lo = out_lo;

    // ---- cross-segment sources: wait for their owners ------------------------
    bool ok = true;
    if (mine && ml > 0 && ms < oend) {
      const uint32_t src_lo = (uint32_t)(ms - off);
      const uint32_t src_hi = (uint32_t)min((uint64_t)src_lo + ml, ms);
      if (src_lo < seg_lo) ok = wait_final(S, c, src_lo, min(src_hi, seg_lo));
    }
    if (__ballot_sync(kFull, !ok)) return;

    if (!long_mode) {
      // ---- owner table -----------------------------------------------------------
      if (mine) {
        const uint32_t a = (uint32_t)(ostart - bs), b = (uint32_t)(oend - bs);
        for (uint32_t i = a; i < b; ++i) W.owner[i] = (uint8_t)lane;
        W.seq_ostart[lane] = a;
        W.seq_ms[lane] = (uint32_t)(ms - bs);
        W.seq_lit[lane] = lit_pos;
        W.seq_off[lane] = off;
      }
      __syncwarp();
      // ---- round 0: every byte whose source is final ----------------------------
      const uint32_t n = be - bs;
      const uint32_t ni = (n + 31) / 32;
      uint32_t pending = 0;
      for (uint32_t i = 0; i < ni; ++i) {
        const uint32_t r = lane + 32 * i;
        if (r >= n) break;
        const uint32_t sq = W.owner[r];
        const uint32_t a = W.seq_ostart[sq], m0 = W.seq_ms[sq];
        uint32_t v;
        if (r < m0) {
          v = byte_at(W.seq_lit[sq] + (r - a));
        } else {
          const uint32_t o = W.seq_off[sq], k = r - m0;
          const uint32_t s = bs + m0 - o + (o > k ? k : k % o);
          if (s >= bs) { pending |= 1u << i; continue; }
          v = exp_of(c.dst, s);
        }
        const uint32_t e = bs + r;
        c.dst[e] = (uint16_t)recombine(__ldg(c.sm + e), v);
      }
      // ---- later rounds: sources produced inside this batch ----------------------
      if (__ballot_sync(kFull, pending != 0)) {
        for (uint32_t round = 0; round < n; ++round) {
          __threadfence_block();
          __syncwarp();
          for (uint32_t i = 0; i < ni; ++i) {
            const unsigned m = __ballot_sync(kFull, (pending >> i) & 1u);
            if (lane == 0) W.pend[i] = m;
          }
          __syncwarp();
          if (__ballot_sync(kFull, pending != 0) == 0) break;
          for (uint32_t i = 0; i < ni; ++i) {
            if (!((pending >> i) & 1u)) continue;
            const uint32_t r = lane + 32 * i;
            const uint32_t sq = W.owner[r];
            const uint32_t m0 = W.seq_ms[sq], o = W.seq_off[sq], k = r - m0;
            const uint32_t sr = m0 - o + (o > k ? k : k % o);  // batch-relative source
            if ((W.pend[sr / 32] >> (sr % 32)) & 1u) continue;
            const uint32_t e = bs + r;
            c.dst[e] = (uint16_t)recombine(__ldg(c.sm + e), exp_of(c.dst, bs + sr));
            pending &= ~(1u << i);
          }
        }
        if (__ballot_sync(kFull, pending != 0)) { set_err(S, kTimeout); return; }
      }
    } else {
      // ---- one sequence longer than kBatchMax: the whole warp copies it ---------
      const uint32_t o0 = (uint32_t)__shfl_sync(kFull, ostart, 0);
      const uint32_t lit_n = (uint32_t)min((uint64_t)__shfl_sync(kFull, ll, 0), (uint64_t)(be - o0));
      const uint32_t lp = __shfl_sync(kFull, lit_pos, 0);
      for (uint32_t i = lane; i < lit_n; i += 32) {
        const uint32_t e = o0 + i;
        c.dst[e] = (uint16_t)recombine(__ldg(c.sm + e), byte_at(lp + i));
      }
      __threadfence_block();
      __syncwarp();
      const uint32_t m0 = o0 + lit_n;
      const uint32_t o = __shfl_sync(kFull, off, 0);
      for (uint32_t k = lane; m0 + k < be; k += 32) {
        const uint32_t s = m0 - o + (o > k ? k : k % o);
        const uint32_t e = m0 + k;
        c.dst[e] = (uint16_t)recombine(__ldg(c.sm + e), exp_of(c.dst, s));
      }
    }
    // ---- publish progress, advance -------------------------------------------------
    __threadfence_block();
    __syncwarp();
    if (lane == 0) *(volatile uint32_t*)&S.frontier[warp] = be;
    ip = __shfl_sync(kFull, seq_end, used - 1);
    op = be;
    if (op < out_hi && ip >= c.src_size) { set_err(S, ZMOE_CHUNK_SHORT_OUTPUT); return; }
  }
}

__global__ void __launch_bounds__(kWarps * 32, 1)
decode_cta_kernel(const zmoe_chunk* __restrict__ chunks, int n_chunks, int32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  CtaSmem& S = *reinterpret_cast<CtaSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const zmoe_chunk d = chunks[blockIdx.x];
  Chunk c;
  c.src = d.src;
  c.sm = d.sm;
  c.dst = d.dst;
  c.index = d.index;
  c.src_size = d.src_size;
  c.out_size = d.out_size;
  c.seg_bytes = d.seg_bytes ? d.seg_bytes : 0xffffffffu;
  c.n_seg = d.index ? d.n_index : 1;
  if (threadIdx.x == 0) {
    S.err = 0;
    if (!c.src || !c.sm || !c.dst || c.src_size == 0 || (c.index && c.n_seg == 0) || (c.index && !d.seg_bytes))
      S.err = ZMOE_CHUNK_BAD_DESC;
  }
  if (threadIdx.x < kWarps) S.frontier[threadIdx.x] = 0;
  __syncthreads();
  WarpSmem& W = S.w[warp];
  if (!S.err && c.out_size > 0) {
    for (uint32_t j = warp; j < c.n_seg; j += kWarps) {
      const uint32_t lo = c.index ? c.seg_out(j) : 0;
      const uint32_t hi = c.index ? c.seg_out(j + 1) : c.out_size;
      const uint32_t in = c.index ? c.seg_in(j) : 0;
      if (lane == 0) *(volatile uint32_t*)&S.frontier[warp] = lo;
      __syncwarp();
      if (lo < hi) decode_segment(S, W, c, in, lo, hi, lane, warp);
      if (cta_failed(S)) break;
    }
    __threadfence_block();
    __syncwarp();
    if (lane == 0) *(volatile uint32_t*)&S.frontier[warp] = c.out_size;
  }
  __syncthreads();
  if (threadIdx.x == 0) status[blockIdx.x] = S.err;
}

}  // namespace

zmoe_status launch_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status, cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  const int smem = (int)sizeof(CtaSmem);
  ZMOE_CUDA_RET(cudaFuncSetAttribute(decode_cta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  decode_cta_kernel<<<n_chunks, kWarps * 32, smem, stream>>>(chunks, n_chunks, status);
  return launch_status("decode_cta_kernel");
}

}  // namespace zmoe
