// LZ4 block encoder on the GPU, hash-chain search in the manner of LZ4HC.
//
// Reference path replaced: LZ4HCcompressor::compress
// (csrc/tensor_engine/compressors.cpp:105-122), i.e. LZ4_compress_HC on one
// CPU thread per exponent chunk, as TensorEngine::PipelineCompress drives it
// when a model is offloaded.  The blocks are valid LZ4 blocks that any LZ4
// decoder (liblz4's LZ4_decompress_safe, this library's decoder) turns back
// into the chunk; they are not byte-identical to liblz4's, whose LZ4HC output
// differs between its own versions too.  Parity is on decoded bytes.
//
// Five launches per call, all chunks at once:
//  1. chain_kernel, one warp per chunk: the hash chains.  The link of
//     position i is i - j for the latest j < i whose 4 bytes hash like those
//     at i (15-bit multiplicative hash), or 0 when there is none within the
//     64 KiB window.  The warp walks the chunk 32 positions at a time; lanes
//     with equal hashes are found with __match_any_sync, so the chains are
//     those of a serial insertion.  The bucket heads sit in shared memory and
//     the source is staged there by cp.async, one 4 KiB block ahead.
//  2. match_kernel, one CTA of 1024 threads per 8192 positions, one thread
//     per position: the longest match among at most max_attempts chain
//     candidates inside the 64 KiB window (the first candidate found wins
//     ties, i.e. the nearest).  The window's links and bytes (217 KB) are
//     staged in shared memory, so every chain step is a shared-memory load.
//     A match may not reach into the block's last 5 bytes, and none starts
//     in its last 12 (the LZ4 end-of-block rules); none crosses a 16 KiB
//     segment boundary.  Each candidate is compared on its first 8 bytes at a
//     fixed cost; only the rare one that shares all 8 goes on byte by byte.
//  3. plan_kernel, scan_kernel, write_kernel: a greedy parse with one step
//     of lazy evaluation (a match is put off by one byte when the next
//     position has a longer one), and the block's bytes: token,
//     literal-length bytes, literals, little-endian offset, match-length
//     bytes, then the last literals.  No match crosses a 16 KiB segment
//     boundary, so one warp parses each segment; a per-chunk scan places the
//     segments' sequences.  Match lengths, offsets and source are staged in
//     shared memory 2048 positions at a time.  A block that would not fit
//     dst_capacity gets size 0 and nothing is written.
//
// No launch waits on another thread or block, so nothing can hang; every
// index is bounded by the chunk's size.  Staging copies whole 16-byte
// granules, so it may read up to 15 bytes before or after a range, inside
// the granules that hold its first and last bytes (never another page).
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kHashLog = 15;
constexpr uint32_t kHashSize = 1u << kHashLog;
constexpr uint32_t kNoHead = 0xFFFFFFFFu;
constexpr uint32_t kMinMatch = 4;
constexpr uint32_t kLastLiterals = 5;                // the last 5 bytes are literals
constexpr uint32_t kMfLimit = 12;                    // no match starts in the last 12 bytes
constexpr uint32_t kMaxOffset = 65535;
constexpr uint32_t kWindow = 65536;
constexpr unsigned kFull = 0xffffffffu;
// A candidate's length is searched up to kLenCap bytes, so that long runs
// cost O(kLenCap) per position; the parse extends a capped match it keeps.
constexpr uint32_t kLenCap = 1024;
// No match crosses a boundary of these segments, so the parse of each one is
// independent of the others (one warp each).
constexpr uint32_t kSegment = 16384;

// The parse's record of one segment.
struct SegRec {
  uint32_t first;                                    // position of its first match (kNoMatch: none)
  uint32_t last_end;                                 // end of its last match
  uint32_t bytes;                                    // its sequences' bytes, but the first one's literals
  uint32_t out_off;                                  // where its sequences start in the block
  uint32_t anchor;                                   // where its first sequence's literals start
  uint32_t pad[3];
};

struct EncChunk {
  const uint8_t* src;
  uint8_t* dst;
  uint16_t* link;                                    // scratch: [src_size] chain links (i - j, 0: none)
  uint16_t* mlen;                                    // scratch: [src_size] best match length (0: none)
  uint16_t* moff;                                    // scratch: [src_size] its offset
  SegRec* seg;                                       // scratch: [nseg] segment records
  uint32_t src_size, dst_capacity, nseg;
};

__device__ __forceinline__ uint32_t hash4(uint32_t v) { return (v * 2654435761u) >> (32 - kHashLog); }

// Scratch: three uint16 arrays of round_up(src_size, 8) entries each, every
// one 16-byte aligned, then one record per segment.
__device__ __forceinline__ EncChunk enc_chunk_of(const zmoe_enc_chunk& d) {
  EncChunk c;
  c.src = d.src;
  c.dst = d.dst;
  const uint64_t n8 = ((uint64_t)d.src_size + 7) & ~7ull;
  uint16_t* base = reinterpret_cast<uint16_t*>(d.scratch);
  c.link = base;
  c.mlen = base + n8;
  c.moff = base + 2 * n8;
  c.seg = reinterpret_cast<SegRec*>(base + 3 * n8);
  c.src_size = d.src_size;
  c.dst_capacity = d.dst_capacity;
  c.nseg = (d.src_size + kSegment - 1) / kSegment;
  return c;
}

// Positions are 32-bit with headroom: chunks above 1 GiB are refused.  An
// empty chunk needs neither source nor scratch.
__device__ __forceinline__ bool bad_enc(const zmoe_enc_chunk& d) {
  return !d.dst || (d.src_size && (!d.src || !d.scratch)) || (reinterpret_cast<uintptr_t>(d.scratch) & 15) != 0 ||
         d.src_size > (1u << 30);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Starts copying the 16-byte granules that cover [g, g + count) to s (16-byte
// aligned, count + 32 bytes); returns the offset of g's first byte in s.
__device__ __forceinline__ uint32_t stage(uint8_t* s, const void* g, uint32_t count, uint32_t tid,
                                          uint32_t nthreads) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(g);
  const uint32_t skew = static_cast<uint32_t>(a & 15);
  if (count == 0) return skew;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a - skew);
  const uint32_t granules = (skew + count + 15) / 16;
  for (uint32_t k = tid; k < granules; k += nthreads) cp_async16(s + 16 * k, base + 16 * k);
  return skew;
}

// 4 bytes at byte offset o of a 4-byte-aligned shared buffer (reads the words
// holding bytes o .. o + 7).
__device__ __forceinline__ uint32_t sload4(const uint8_t* s, uint32_t o) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(s) + (o >> 2);
  return __funnelshift_r(w[0], w[1], (o & 3) * 8);
}

// ---------------------------------------------------------------------------
// 1. hash chains (one warp per chunk)
// ---------------------------------------------------------------------------
constexpr uint32_t kChainBlock = 4096;               // positions per staged block
constexpr uint32_t kChainBuf = kChainBlock + 64;     // bytes per staging buffer
constexpr int kChainSmem = (int)(kHashSize * sizeof(uint32_t) + 2 * kChainBuf);

__global__ void __launch_bounds__(32) chain_kernel(const zmoe_enc_chunk* __restrict__ chunks) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* head = reinterpret_cast<uint32_t*>(smem);   // [kHashSize] latest position per bucket
  uint8_t* buf = smem + kHashSize * sizeof(uint32_t);    // [2][kChainBuf] source blocks
  const zmoe_enc_chunk d = chunks[blockIdx.x];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  const uint32_t lane = threadIdx.x;
  const uint32_t n = c.src_size;
  for (uint32_t h = lane; h < kHashSize; h += 32) head[h] = kNoHead;
  // bytes a block needs: its positions and the 3 after the last one
  uint32_t skew = stage(buf, c.src, min(n, kChainBlock + 3), lane, 32);
  cp_async_commit();
  const uint32_t lt = lane == 0 ? 0u : (kFull >> (32 - lane));   // lanes below this one
  uint32_t b = 0;
  for (uint32_t b0 = 0; b0 < n; b0 += kChainBlock, b ^= 1) {
    const uint32_t nb0 = b0 + kChainBlock;
    uint32_t skew_next = 0;
    if (nb0 < n) skew_next = stage(buf + (b ^ 1) * kChainBuf, c.src + nb0, min(n - nb0, kChainBlock + 3), lane, 32);
    cp_async_commit();
    cp_async_wait<1>();                              // this block's copy is complete
    __syncwarp();
    const uint8_t* sb = buf + b * kChainBuf;
    const uint32_t b1 = min(n, nb0);
    for (uint32_t i0 = b0; i0 < b1; i0 += 32) {
      const uint32_t i = i0 + lane;
      const bool keyed = i + kMinMatch <= n;         // has 4 bytes to hash
      const uint32_t h = keyed ? hash4(sload4(sb, skew + (i - b0))) : kHashSize + lane;   // unkeyed lanes match no one
      const uint32_t peers = __match_any_sync(kFull, h);
      const uint32_t below = peers & lt;
      uint32_t j = kNoHead;
      if (keyed) j = below ? i0 + (31 - __clz(below)) : head[h];
      __syncwarp();                                  // every read of head before the writes
      if (keyed && (peers >> lane) == 1u) head[h] = i;   // the highest lane of its bucket
      if (i < n) c.link[i] = (uint16_t)(j != kNoHead && i - j <= kMaxOffset ? i - j : 0u);
      __syncwarp();
    }
    skew = skew_next;
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// 2. longest match per position (one CTA per 8192 positions)
// ---------------------------------------------------------------------------
constexpr uint32_t kMatchBlock = 8192;               // positions per CTA
constexpr uint32_t kMatchThreads = 1024;
constexpr uint32_t kLinkStage = kWindow + kMatchBlock;                  // link entries staged
constexpr uint32_t kSrcStage = kWindow + kMatchBlock + kLenCap + 64;    // source bytes staged (with skew, slack)
constexpr int kMatchSmem = (int)(kLinkStage * 2 + kSrcStage);           // 222,272 bytes

// Chunks are walked block by block in a grid-stride loop over gridDim.x, so
// the launch needs no chunk sizes.  Block p0 stages links [lo, p1) and bytes
// [lo, min(n, p1 + kLenCap)), lo = max(0, p0 - 65536): every candidate of a
// position in [p0, p1) and every byte a match compares lies inside.
__global__ void __launch_bounds__(kMatchThreads, 1) match_kernel(const zmoe_enc_chunk* __restrict__ chunks,
                                                                 int max_attempts) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* slink = reinterpret_cast<uint16_t*>(smem);
  uint8_t* ssrc = smem + kLinkStage * 2;
  const zmoe_enc_chunk d = chunks[blockIdx.y];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  const uint32_t n = c.src_size;
  const uint32_t tid = threadIdx.x;
  for (uint32_t p0 = blockIdx.x * kMatchBlock; p0 < n; p0 += gridDim.x * kMatchBlock) {
    const uint32_t p1 = min(n, p0 + kMatchBlock);
    const uint32_t lo = p0 > kWindow ? p0 - kWindow : 0u;   // a multiple of 16 entries: 16-byte aligned
    const uint32_t hi = min(n, p1 + kLenCap);
    __syncthreads();                                 // the previous block's reads are done
    stage(reinterpret_cast<uint8_t*>(slink), c.link + lo, (p1 - lo) * 2, tid, kMatchThreads);
    const uint32_t skew = stage(ssrc, c.src + lo, hi - lo, tid, kMatchThreads);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(ssrc);
    for (uint32_t i = p0 + tid; i < p1; i += kMatchThreads) {
      uint32_t best = 0, best_off = 0;
      const uint32_t seg_end = min(n, (i / kSegment + 1) * kSegment);
      if (i + kMfLimit <= n && seg_end - i >= kMinMatch) {   // a match may start here
        const uint32_t max_len = min(min(n - kLastLiterals - i, kLenCap), seg_end - i);
        const uint32_t oi = skew + (i - lo);
        // Every candidate is compared on its first 8 bytes at a fixed cost (the
        // position's own 8 bytes sit in registers); only one that shares all 8
        // and may beat the best goes on byte by byte (about 0.2% of them in
        // BF16 exponent data), so the lanes of a warp rarely part ways.
        const uint32_t own0 = sload4(ssrc, oi), own1 = sload4(ssrc, oi + 4);
        uint32_t cand = i;
        uint32_t step = slink[i - lo];
        for (int a = 0; a < max_attempts && step != 0; ++a) {
          cand -= step;
          if (i - cand > kMaxOffset) break;          // farther links are out of the window too
          const uint32_t oc = skew + (cand - lo);
          const uint32_t* w = sw + (oc >> 2);
          const uint32_t sh = (oc & 3) * 8;
          const uint32_t w1 = w[1];
          const uint32_t d0 = __funnelshift_r(w[0], w1, sh) ^ own0;
          const uint32_t d1 = __funnelshift_r(w1, w[2], sh) ^ own1;
          uint32_t len = d0 ? (uint32_t)(__ffs(d0) - 1) >> 3 : d1 ? 4 + ((uint32_t)(__ffs(d1) - 1) >> 3) : 8u;
          if (len == 8 && max_len > 8 && (best < 8 || ssrc[oc + best] == ssrc[oi + best])) {
            while (len < max_len) {                  // 4 bytes at a time; bytes past max_len are cut below
              const uint32_t x = sload4(ssrc, oc + len) ^ sload4(ssrc, oi + len);
              if (x) {
                len += (uint32_t)(__ffs(x) - 1) >> 3;
                break;
              }
              len += 4;
            }
          }
          len = min(len, max_len);
          if (len >= kMinMatch && len > best) {
            best = len;
            best_off = i - cand;
            if (len >= max_len) break;
          }
          step = slink[cand - lo];
        }
      }
      c.mlen[i] = (uint16_t)(best >= kMinMatch ? best : 0u);
      c.moff[i] = (uint16_t)best_off;
    }
  }
}

// ---------------------------------------------------------------------------
// 3. parse and write the block: plan (one warp per segment), scan (one warp
//    per chunk), write (one warp per segment)
// ---------------------------------------------------------------------------
// A segment's sequences are those whose match starts in it.  The plan pass
// sizes them all but the literal part of the first, whose literals start at
// the end of the last match of an earlier segment; the scan fixes that start
// (the anchor) and each segment's output offset, checks the capacity and
// writes the block's last literals; the write pass parses again and writes.
constexpr uint32_t kNoMatch = 0xFFFFFFFFu;
constexpr uint32_t kParseBlock = 2048;               // positions staged at a time
constexpr uint32_t kParseStage = kParseBlock + 40;   // entries staged: a window of 32 and its successor past the block
constexpr uint32_t kParseBuf = kParseStage * 2 + 32; // bytes per uint16 buffer
constexpr int kParseSmem = (int)(2 * kParseBuf + kParseStage + 64);

// The staged source: bytes [blk0, stop) of the chunk at s + skew; others are
// read from global memory.
struct Staged {
  const uint8_t* g;
  const uint8_t* s;
  uint32_t skew, blk0, stop;
  __device__ __forceinline__ uint8_t at(uint32_t pos) const {
    return pos >= blk0 && pos < stop ? s[skew + (pos - blk0)] : g[pos];
  }
};

// Bytes of the 255-run that follows a length nibble of 15 (rest = length - 15).
__device__ __forceinline__ uint32_t run_bytes(uint32_t rest) { return rest / 255 + 1; }
__device__ __forceinline__ uint32_t lit_bytes(uint32_t ll) { return ll + (ll >= 15 ? run_bytes(ll - 15) : 0u); }
__device__ __forceinline__ uint32_t match_bytes(uint32_t ml) {
  return 2 + (ml - kMinMatch >= 15 ? run_bytes(ml - kMinMatch - 15) : 0u);
}

// rest as a 255-run at dst, the lanes striding over its bytes.
__device__ __forceinline__ void put_run(uint8_t* dst, uint32_t rest, uint32_t lane) {
  const uint32_t nb = rest / 255;
  for (uint32_t k = lane; k <= nb; k += 32) dst[k] = k < nb ? (uint8_t)255 : (uint8_t)(rest - nb * 255);
}

// One sequence at dst: token, literal-length run, the literals
// [anchor, anchor + ll), little-endian offset, match-length run; ml == 0 is
// the block's last literals (no match part).  Returns its size.  Every
// argument is the same in all lanes; the caller has checked the capacity.
__device__ uint32_t put_sequence(uint8_t* dst, const Staged& src, uint32_t anchor, uint32_t ll, uint32_t off,
                                 uint32_t ml, uint32_t lane) {
  const uint32_t mcode = ml ? ml - kMinMatch : 0u;
  const uint32_t llb = ll >= 15 ? run_bytes(ll - 15) : 0u;
  if (lane == 0) dst[0] = (uint8_t)(((ll >= 15 ? 15u : ll) << 4) | (ml ? (mcode >= 15 ? 15u : mcode) : 0u));
  if (llb) put_run(dst + 1, ll - 15, lane);
  uint8_t* q = dst + 1 + llb;
  for (uint32_t k = lane; k < ll; k += 32) q[k] = src.at(anchor + k);
  if (!ml) return 1 + llb + ll;
  q += ll;
  if (lane == 0) {
    q[0] = (uint8_t)(off & 0xFF);
    q[1] = (uint8_t)(off >> 8);
  }
  if (mcode >= 15) put_run(q + 2, mcode - 15, lane);
  return 1 + llb + ll + match_bytes(ml);
}

// Parses segment k: positions visited in order, a window of 32 tested at
// once, and the first position the serial parse would take found with a
// ballot (a match of at least 4 whose successor, if it may start a match, is
// not longer).  WRITE = false records the segment's plan; WRITE = true writes
// its sequences at the offset the scan assigned.
template <bool WRITE>
__device__ void parse_segment(const EncChunk& c, uint32_t k, uint8_t* smem, uint32_t lane) {
  uint16_t* sl = reinterpret_cast<uint16_t*>(smem);              // staged match lengths
  uint16_t* so = reinterpret_cast<uint16_t*>(smem + kParseBuf);  // staged offsets
  uint8_t* ss = smem + 2 * kParseBuf;                             // staged source
  const uint32_t n = c.src_size;
  const uint32_t e = min(n, (k + 1) * kSegment);
  uint32_t anchor = 0, op = 0;
  if (WRITE) {
    op = c.seg[k].out_off;
    anchor = c.seg[k].anchor;
    if (op == kNoMatch) return;                      // no match here, or the block did not fit
  }
  Staged src{c.src, ss, 0u, 0u, 0u};
  bool have = false;                                 // a block is staged
  uint32_t first = kNoMatch, bytes = 0;
  uint32_t i = k * kSegment;
  while (i < e && i + kMfLimit <= n) {
    if (!have || i >= src.blk0 + kParseBlock) {      // stage the block that starts at i (rounded down to 8)
      __syncwarp();                                  // the previous block's reads are done
      const uint32_t b0 = i & ~7u;
      const uint32_t cnt = min(n - b0, kParseStage);
      stage(reinterpret_cast<uint8_t*>(sl), c.mlen + b0, cnt * 2, lane, 32);
      stage(reinterpret_cast<uint8_t*>(so), c.moff + b0, cnt * 2, lane, 32);
      src.skew = stage(ss, c.src + b0, cnt, lane, 32);
      cp_async_commit();
      cp_async_wait<0>();
      __syncwarp();
      src.blk0 = b0;
      src.stop = b0 + cnt;
      have = true;
    }
    const uint32_t j = i + lane;
    uint32_t len = 0;
    bool take = false;
    if (j < e && j + kMfLimit <= n) {
      len = sl[j - src.blk0];
      if (len >= kMinMatch)                          // lazy: put off when the next is longer
        take = !(j + 1 < e && j + 1 + kMfLimit <= n && sl[j + 1 - src.blk0] > len);
    }
    const uint32_t taken = __ballot_sync(kFull, take);
    if (!taken) {
      i += 32;
      continue;
    }
    const uint32_t f = __ffs(taken) - 1;
    uint32_t ml = __shfl_sync(kFull, len, f);
    i += f;
    const uint32_t off = so[i - src.blk0];
    if (ml == kLenCap) {                             // capped in the search: extend it here
      const uint32_t end = min(n - kLastLiterals, e);
      for (;;) {
        const uint32_t p = i + ml + lane;
        const uint32_t stop = __ballot_sync(kFull, p >= end || c.src[p] != c.src[p - off]);
        if (stop) {
          ml += __ffs(stop) - 1;
          break;
        }
        ml += 32;
      }
    }
    if (WRITE) {
      op += put_sequence(c.dst + op, src, anchor, i - anchor, off, ml, lane);
    } else if (first == kNoMatch) {
      first = i;
      bytes = 1 + match_bytes(ml);                   // its literal part is sized by the scan
    } else {
      bytes += 1 + lit_bytes(i - anchor) + match_bytes(ml);
    }
    i += ml;
    anchor = i;
  }
  if (!WRITE && lane == 0) {
    SegRec& r = c.seg[k];
    r.first = first;
    r.last_end = anchor;
    r.bytes = bytes;
  }
}

__global__ void __launch_bounds__(32) plan_kernel(const zmoe_enc_chunk* __restrict__ chunks) {
  extern __shared__ __align__(16) uint8_t smem[];
  const zmoe_enc_chunk d = chunks[blockIdx.y];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  for (uint32_t k = blockIdx.x; k < c.nseg; k += gridDim.x) parse_segment<false>(c, k, smem, threadIdx.x);
}

__global__ void __launch_bounds__(32) write_kernel(const zmoe_enc_chunk* __restrict__ chunks) {
  extern __shared__ __align__(16) uint8_t smem[];
  const zmoe_enc_chunk d = chunks[blockIdx.y];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  for (uint32_t k = blockIdx.x; k < c.nseg; k += gridDim.x) parse_segment<true>(c, k, smem, threadIdx.x);
}

__global__ void __launch_bounds__(32) scan_kernel(const zmoe_enc_chunk* __restrict__ chunks,
                                                  uint32_t* __restrict__ out_sizes) {
  const zmoe_enc_chunk d = chunks[blockIdx.x];
  const uint32_t lane = threadIdx.x;
  if (bad_enc(d)) {
    if (lane == 0) out_sizes[blockIdx.x] = 0;
    return;
  }
  const EncChunk c = enc_chunk_of(d);
  const uint32_t n = c.src_size;
  uint64_t op = 0;
  uint32_t prev_end = 0;
  if (lane == 0) {
    for (uint32_t k = 0; k < c.nseg; ++k) {
      SegRec& r = c.seg[k];
      if (r.first == kNoMatch) {
        r.out_off = kNoMatch;
        continue;
      }
      r.anchor = prev_end;
      r.out_off = (uint32_t)min(op, (uint64_t)kNoMatch - 1);
      op += r.bytes + lit_bytes(r.first - prev_end);
      prev_end = r.last_end;
    }
    op += 1 + lit_bytes(n - prev_end);               // the last literals
  }
  op = __shfl_sync(kFull, op, 0);
  prev_end = __shfl_sync(kFull, prev_end, 0);
  const bool ok = op <= c.dst_capacity;
  if (!ok) {                                         // nothing is written
    for (uint32_t k = lane; k < c.nseg; k += 32) c.seg[k].out_off = kNoMatch;
  } else {
    const Staged g{c.src, nullptr, 0u, 0u, 0u};
    const uint32_t tail = 1 + lit_bytes(n - prev_end);
    put_sequence(c.dst + (op - tail), g, prev_end, n - prev_end, 0, 0, lane);
  }
  if (lane == 0) out_sizes[blockIdx.x] = ok ? (uint32_t)op : 0u;
}

}  // namespace

zmoe_status launch_encode_chunks(const zmoe_enc_chunk* chunks, int n_chunks, int max_attempts, uint32_t* out_sizes,
                                 cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  ZMOE_CHECK_ARG(n_chunks <= 65535, "lz4_encode: %d chunks in one launch (at most 65535)", n_chunks);
  ZMOE_CHECK_ARG(max_attempts >= 1 && max_attempts <= 65536, "lz4_encode: max_attempts=%d outside [1, 65536]",
                 max_attempts);
  static uint64_t attr_set = 0;                      // devices whose attributes are set
  int dev = 0;
  ZMOE_CUDA_RET(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << (dev & 63)))) {
    ZMOE_CUDA_RET(cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kChainSmem));
    ZMOE_CUDA_RET(cudaFuncSetAttribute(match_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMatchSmem));
    attr_set |= 1ull << (dev & 63);
  }
  chain_kernel<<<n_chunks, 32, kChainSmem, stream>>>(chunks);
  zmoe_status st = launch_status("chain_kernel");
  if (st != ZMOE_OK) return st;
  // grid-stride over blocks and segments: 128 blocks of 8192 positions and 64
  // segments of 16 KiB cover a 1 MiB chunk in one pass; larger chunks loop
  match_kernel<<<dim3(128, n_chunks), kMatchThreads, kMatchSmem, stream>>>(chunks, max_attempts);
  if ((st = launch_status("match_kernel")) != ZMOE_OK) return st;
  plan_kernel<<<dim3(64, n_chunks), 32, kParseSmem, stream>>>(chunks);
  if ((st = launch_status("plan_kernel")) != ZMOE_OK) return st;
  scan_kernel<<<n_chunks, 32, 0, stream>>>(chunks, out_sizes);
  if ((st = launch_status("scan_kernel")) != ZMOE_OK) return st;
  write_kernel<<<dim3(64, n_chunks), 32, kParseSmem, stream>>>(chunks);
  return launch_status("write_kernel");
}

}  // namespace zmoe

// three uint16 arrays (chain link, match length, match offset) of
// round_up(src_size, 8) entries, then 32 bytes per 16 KiB segment
extern "C" uint64_t zmoe_lz4_encode_scratch_bytes(uint32_t src_size) {
  const uint64_t segments = src_size ? ((uint64_t)src_size + 16383) / 16384 : 1;
  return 6 * (((uint64_t)src_size + 7) & ~7ull) + 32 * segments;
}
