// Fused LZ4-block decode + plane recombine (sm_100a).
//
// Reference path replaced: per exponent chunk, LZ4_decompress_safe_partial
// on a CPU worker (csrc/tensor_engine/compressors.cpp:195-211, driven by
// tensor_engine.cpp:421-474), a memcpy into a pinned dock, then the recombine
// kernel (csrc/kernels/tensor_recover.cu:12-43) reading both planes over
// zero-copy host memory.
//
// Here one warp owns one LZ4 block (one exponent chunk).  The warp walks the
// block in batches of up to 32 sequences:
//
//  1. 256 compressed bytes from the current token position are staged in
//     shared memory; every lane computes, for 8 byte positions, where the next
//     token would start if a token started there (`next_token`).
//  2. Pointer doubling over that table (5 levels) gives lane l the start of
//     sequence l of the batch in O(log 32) shared-memory lookups, so the
//     serial token chain is resolved by the whole warp at once.
//  3. Each lane decodes its own sequence header; a warp scan turns sequence
//     lengths into output positions.
//  4. Literals are written first (lane-serial when short, warp-cooperative when
//     long).  Matches then run in dependency rounds: a match whose source
//     overlaps the match output of an earlier, unfinished lane of the same
//     batch waits for the next round; everything before the batch is complete.
//     A match copy reads source byte (start - off + i mod off), which resolves
//     overlapping copies without a serial loop.
//  5. Every decoded exponent byte is merged with its sign+mantissa byte and
//     stored as BF16 directly in the destination slot.  Match sources are read
//     back from the BF16 slot (exponent = bits 7..14) through L2.
//
// Errors (zero or out-of-range offsets, lengths running past the block, a block
// that ends short of out_size) set the chunk's status word; the kernel never
// traps.  Output past out_size is clipped and decoding stops there, the
// targetOutputSize = out_size behaviour of LZ4_decompress_safe_partial.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr uint32_t kWin = 256;       // compressed bytes staged per batch
constexpr int kLevels = 5;           // doubling tables: jumps of 1,2,4,8,16 tokens
constexpr int kWarpsPerBlock = 4;
constexpr uint32_t kLong = 32;       // lengths above this are copied by the whole warp
constexpr unsigned kFull = 0xffffffffu;

struct WarpSmem {
  uint8_t win[kWin];
  uint16_t jump[kLevels][kWin];
};

// Start of the token following a token at window position i, or kWin when the
// chain cannot continue inside the window (the token is the block's last
// sequence, a length runs past the staged bytes, or i is outside the data).
__device__ __forceinline__ uint32_t next_token(const uint8_t* win, uint32_t i, uint32_t avail,
                                               uint32_t rem) {
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
  if (j >= rem) return kWin;         // literals reach the block end: last sequence
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

__device__ __forceinline__ uint32_t byte_at(const uint8_t* __restrict__ src, const uint8_t* win,
                                            uint32_t base, uint32_t avail, uint32_t pos) {
  const uint32_t rel = pos - base;
  return rel < avail ? (uint32_t)win[rel] : (uint32_t)__ldg(src + pos);
}

__device__ __forceinline__ uint32_t exp_of(const uint16_t* dst, uint64_t pos) {
  return ((uint32_t)__ldcg(dst + pos) >> 7) & 0xFFu;
}

__global__ void __launch_bounds__(kWarpsPerBlock * 32)
decode_warp_kernel(const zmoe_chunk* __restrict__ chunks, int n_chunks, int32_t* __restrict__ status) {
  __shared__ WarpSmem smem_all[kWarpsPerBlock];
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int ci = blockIdx.x * kWarpsPerBlock + warp;
  if (ci >= n_chunks) return;
  WarpSmem& S = smem_all[warp];

  const zmoe_chunk c = chunks[ci];
  const uint8_t* __restrict__ src = c.src;
  const uint8_t* __restrict__ sm = c.sm;
  uint16_t* dst = c.dst;
  const uint32_t src_size = c.src_size;
  const uint32_t out_size = c.out_size;

  int32_t err = ZMOE_CHUNK_OK;
  if (src == nullptr || sm == nullptr || dst == nullptr || src_size == 0) err = ZMOE_CHUNK_BAD_DESC;
  uint32_t ip = 0;
  uint64_t op = 0;
  bool finished = (err != ZMOE_CHUNK_OK) || out_size == 0;

  while (!finished) {
    if (ip >= src_size) {                      // block ended right after a match
      err = ZMOE_CHUNK_INPUT_OVERRUN;
      break;
    }
    const uint32_t rem = src_size - ip;
    const uint32_t avail = rem < kWin ? rem : kWin;
    for (uint32_t b = lane; b < kWin; b += 32) S.win[b] = b < avail ? __ldg(src + ip + b) : 0;
    __syncwarp();
#pragma unroll
    for (uint32_t q = 0; q < kWin / 32; ++q) {
      const uint32_t i = lane * (kWin / 32) + q;
      S.jump[0][i] = (uint16_t)next_token(S.win, i, avail, rem);
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k + 1 < kLevels; ++k) {
#pragma unroll
      for (uint32_t q = 0; q < kWin / 32; ++q) {
        const uint32_t i = lane * (kWin / 32) + q;
        const uint32_t v = S.jump[k][i];
        S.jump[k + 1][i] = v < kWin ? S.jump[k][v] : (uint16_t)kWin;
      }
      __syncwarp();
    }
    uint32_t p = 0;
#pragma unroll
    for (int k = 0; k < kLevels; ++k)
      if ((lane >> k) & 1) p = p < kWin ? S.jump[k][p] : kWin;
    const bool valid = p < avail;

    // ---- decode this lane's sequence header --------------------------------
    uint64_t ll = 0, ml = 0;
    uint32_t off = 0, lit_pos = 0, seq_end = 0;
    bool last = false;
    int lerr = 0;
    if (valid) {
      const uint32_t tok = S.win[p];
      uint32_t q = ip + p + 1;
      ll = tok >> 4;
      if (ll == 15) {
        uint32_t b;
        do {
          if (q >= src_size) { lerr = ZMOE_CHUNK_INPUT_OVERRUN; break; }
          b = byte_at(src, S.win, ip, avail, q++);
          ll += b;
        } while (b == 255);
      }
      lit_pos = q;
      if (!lerr) {
        if ((uint64_t)q + ll > src_size) {
          lerr = ZMOE_CHUNK_INPUT_OVERRUN;
        } else {
          q += (uint32_t)ll;
          if (q == src_size) {
            last = true;
          } else if (q + 2 > src_size) {
            lerr = ZMOE_CHUNK_INPUT_OVERRUN;
          } else {
            off = byte_at(src, S.win, ip, avail, q) | (byte_at(src, S.win, ip, avail, q + 1) << 8);
            q += 2;
            ml = tok & 15;
            if (ml == 15) {
              uint32_t b;
              do {
                if (q >= src_size) { lerr = ZMOE_CHUNK_INPUT_OVERRUN; break; }
                b = byte_at(src, S.win, ip, avail, q++);
                ml += b;
              } while (b == 255);
            }
            ml += 4;
          }
        }
      }
      seq_end = q;
    }
    const unsigned vmask = __ballot_sync(kFull, valid);
    const int count = __popc(vmask);

    // ---- output positions ----------------------------------------------------
    const uint64_t len = (valid && !lerr) ? ll + ml : 0;
    uint64_t incl = len;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint64_t v = __shfl_up_sync(kFull, incl, d);
      if (lane >= (uint32_t)d) incl += v;
    }
    const uint64_t ostart = op + incl - len;
    // clip to the target size (partial decode semantics)
    const uint64_t lit_n = valid ? (ostart >= out_size ? 0 : min(ll, out_size - ostart)) : 0;
    const uint64_t ms = ostart + ll;
    const uint64_t mlen = (valid && ml > 0 && ms < out_size) ? min(ml, out_size - ms) : 0;
    if (valid && !lerr && mlen > 0 && (off == 0 || off > ms)) lerr = ZMOE_CHUNK_BAD_OFFSET;
    // Lanes after the first one that reaches the target never execute.
    const unsigned reach = __ballot_sync(kFull, valid && ostart + len >= out_size);
    const int stop_lane = reach ? __ffs(reach) - 1 : 31;
    const unsigned emask = __ballot_sync(kFull, lerr != 0) & (stop_lane == 31 ? kFull : ((2u << stop_lane) - 1));
    if (emask) {
      err = __shfl_sync(kFull, lerr, __ffs(emask) - 1);
      break;
    }
    const bool live = valid && (int)lane <= stop_lane;

    // ---- literals -------------------------------------------------------------
    if (live && lit_n > 0 && lit_n <= kLong) {
      for (uint32_t i = 0; i < (uint32_t)lit_n; ++i) {
        const uint64_t e = ostart + i;
        dst[e] = (uint16_t)recombine(__ldg(sm + e), byte_at(src, S.win, ip, avail, lit_pos + i));
      }
    }
    unsigned lmask = __ballot_sync(kFull, live && lit_n > kLong);
    while (lmask) {
      const int j = __ffs(lmask) - 1;
      lmask &= lmask - 1;
      const uint64_t o = __shfl_sync(kFull, ostart, j);
      const uint64_t n = __shfl_sync(kFull, lit_n, j);
      const uint32_t lp = __shfl_sync(kFull, lit_pos, j);
      for (uint64_t i = lane; i < n; i += 32)
        dst[o + i] = (uint16_t)recombine(__ldg(sm + o + i), byte_at(src, S.win, ip, avail, lp + (uint32_t)i));
    }
    __threadfence_block();
    __syncwarp();

    // ---- matches, in dependency rounds ----------------------------------------
    const bool need = live && mlen > 0;
    const uint64_t me = need ? ms + mlen : 0;
    const uint64_t src_lo = need ? ms - off : 0;
    const uint64_t src_hi = need ? min(src_lo + mlen, ms) : 0;
    unsigned dep = 0;
    for (int j = 0; j < 32; ++j) {
      const uint64_t msj = __shfl_sync(kFull, ms, j);
      const uint64_t mej = __shfl_sync(kFull, me, j);
      if (need && j < (int)lane && mej > src_lo && msj < src_hi) dep |= 1u << j;
    }
    bool done = !need;
    for (int round = 0; round <= 32; ++round) {
      const unsigned done_mask = __ballot_sync(kFull, done);
      if (done_mask == kFull) break;
      const bool ready = !done && (dep & ~done_mask) == 0;
      if (ready && mlen <= kLong) {
        for (uint32_t i = 0; i < (uint32_t)mlen; ++i) {
          const uint64_t e = ms + i;
          const uint64_t s = src_lo + (off > i ? i : i % off);
          dst[e] = (uint16_t)recombine(__ldg(sm + e), exp_of(dst, s));
        }
        done = true;
      }
      unsigned cmask = __ballot_sync(kFull, ready && mlen > kLong);
      while (cmask) {
        const int j = __ffs(cmask) - 1;
        cmask &= cmask - 1;
        const uint64_t m0 = __shfl_sync(kFull, ms, j);
        const uint64_t n = __shfl_sync(kFull, mlen, j);
        const uint32_t o = __shfl_sync(kFull, off, j);
        for (uint64_t i = lane; i < n; i += 32) {
          const uint64_t s = m0 - o + (o > i ? i : i % o);
          dst[m0 + i] = (uint16_t)recombine(__ldg(sm + m0 + i), exp_of(dst, s));
        }
        if ((int)lane == j) done = true;
      }
      __threadfence_block();
      __syncwarp();
    }

    // ---- advance ----------------------------------------------------------------
    const int tail = min(count - 1, stop_lane);
    ip = __shfl_sync(kFull, seq_end, tail);
    op = min(op + __shfl_sync(kFull, incl, tail), (uint64_t)out_size);
    const bool ended = __ballot_sync(kFull, live && last) != 0;
    if (op >= out_size) {
      finished = true;
    } else if (ended) {
      err = ZMOE_CHUNK_SHORT_OUTPUT;
      finished = true;
    }
  }
  if (lane == 0) status[ci] = err;
}

}  // namespace

zmoe_status launch_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status,
                                 cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  const int blocks = (n_chunks + kWarpsPerBlock - 1) / kWarpsPerBlock;
  decode_warp_kernel<<<blocks, kWarpsPerBlock * 32, 0, stream>>>(chunks, n_chunks, status);
  return launch_status("decode_warp_kernel");
}

}  // namespace zmoe
