// Fused LZ4-block decode + plane recombine (sm_100a).
//
// Reference path replaced: per exponent chunk, LZ4_decompress_safe_partial
// on a CPU worker (csrc/tensor_engine/compressors.cpp:195-211, driven by
// tensor_engine.cpp:421-474), a memcpy into a pinned dock, then the recombine
// kernel (csrc/kernels/tensor_recover.cu:12-43) reading both planes over
// zero-copy host memory.
//
// One CTA of 6 warps decodes one LZ4 block.  LZ4HC matches chain back through
// earlier matches (median offset ~20 KB), so the data dependencies of a block
// are nearly serial; parsing the token stream is not.  The work is split so
// that only a cheap gather stays serial:
//
//  * 4 parser warps.  A segment index built at load time (zmoe_lz4_build_index:
//    the first sequence at or after every 1 KiB of output) lets parser p take
//    segments p, p+4, ...  A parser looks at 255 compressed bytes (prefetched
//    into shared memory with cp.async), builds a next-token table in
//    registers (8 positions per lane, packed bytes) and finds up to 32 token
//    starts at once by pointer doubling with warp shuffles; it decodes the
//    headers and turns a batch of up to 256 output bytes into one 32-bit
//    descriptor per output byte — a literal value, or the absolute position
//    of its source byte — with bytes spread over lanes by position (owner
//    sequence from a bitmap of sequence starts).  Sources inside the batch
//    itself (short offsets, overlapping copies) are chased at parse time until
//    they reach a literal or a byte before the batch, so a descriptor never
//    depends on its batch.  All of this keeps shared-memory traffic low: the
//    decoder's limit is shared-memory wavefronts, not HBM.
//    Batches go to a 6-slot queue per parser (one whole segment).
//  * 1 resolver warp.  It takes the batches in output order and, per byte,
//    reads either the literal or ring[source & 0xFFFF] from a 64 KiB
//    shared-memory window of decoded exponents (LZ4 offsets are < 64 KiB),
//    then writes the batch into the window: one gather + one scatter per
//    byte, no dependency waits.  A sequence longer than a batch is copied by
//    the whole warp 32 bytes at a time from its most recent equal byte.
//  * 1 flusher warp.  It follows the resolver through the window, merges 16
//    exponent bytes with 16 sign+mantissa bytes (128-bit loads) into BF16 and
//    stores 32 bytes per lane; the resolver never overwrites a window byte the
//    flusher has not consumed.
//
// Roles synchronise through counters in shared memory; every wait is bounded
// and gives up with an error status.  Errors (bad offsets, lengths past the
// block, a block ending short of out_size) set the chunk's status word; the
// kernel never traps.  Output past out_size is clipped (the targetOutputSize
// = out_size behaviour of LZ4_decompress_safe_partial).
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kParsers = 4;
constexpr int kWarps = kParsers + 2;          // parsers, resolver, flusher
constexpr int kResolver = kParsers;           // warp kParsers + 1 is the flusher
constexpr int kSlots = 6;                     // queue depth per parser (a 1 KiB segment)
constexpr uint32_t kWin = 256;                // compressed bytes staged per parse step
constexpr uint32_t kInBuf = 1024;             // prefetched compressed bytes per segment buffer
constexpr int kLevels = 5;                    // jumps of 1, 2, 4, 8, 16 tokens
constexpr uint32_t kStop = 255;               // next-token entry: chain stops (window positions 0..254)
constexpr uint32_t kBatch = 256;              // output bytes of one batch
constexpr uint32_t kRing = 65536;             // decoded-exponent window
constexpr uint32_t kRingMask = kRing - 1;
constexpr uint32_t kLit = 0x80000000u;        // descriptor: literal value in bits 0..7
constexpr uint32_t kInternal = 0x40000000u;   // descriptor (parse time only): batch-relative source
constexpr long long kSpinCycles = 2000000000LL;   // ~1 s at 1.9 GHz
constexpr unsigned kFull = 0xffffffffu;
constexpr int32_t kTimeout = 5;

struct Slot {
  uint32_t desc[kBatch];
  uint32_t bs, n, mode, pad;                  // mode 0: descriptors, 1: one long sequence
  uint32_t l_ll, l_lit, l_ml, l_off;          // long sequence: literal count/source, match length/offset
};

struct ParserSmem {
  __align__(16) uint8_t inbuf[2][kInBuf];
  uint32_t winw[kWin / 4 + 2];
  Slot slot[kSlots];
};

struct Smem {
  uint8_t ring[kRing];
  ParserSmem ps[kParsers];
  uint32_t q_tail[kParsers];
  uint32_t q_head[kParsers];
  uint32_t res_pos;                           // bytes [0, res_pos) resolved into the ring
  uint32_t flush_pos;                         // bytes [0, flush_pos) consumed by the flusher
  int32_t err;
};

struct Chunk {
  const uint8_t* src;
  const uint8_t* sm;
  uint16_t* dst;
  const uint32_t* index;
  uint32_t src_size, out_size, n_seg;
  uint32_t rofs;   // ring index of position i is (i + rofs) & kRingMask; makes 16-byte
                   // groups that the flusher loads aligned both in the ring and in memory

  __device__ __forceinline__ uint32_t ri(uint32_t pos) const { return (pos + rofs) & kRingMask; }
  __device__ uint32_t seg_out(uint32_t j) const {
    if (j >= n_seg) return out_size;
    if (!index) return 0;
    return min(__ldg(index + 2 * j + 1), out_size);
  }
  __device__ uint32_t seg_in(uint32_t j) const { return index ? __ldg(index + 2 * j) : 0; }
};

__device__ __forceinline__ uint32_t vload(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void vstore(uint32_t* p, uint32_t v) { *(volatile uint32_t*)p = v; }
__device__ __forceinline__ bool failed(Smem& S) { return *(volatile int32_t*)&S.err != 0; }
__device__ __forceinline__ void set_err(Smem& S, int32_t code) { atomicCAS(&S.err, 0, code); }

// Spin (bounded) until cond() holds; false on error or timeout.
template <class F>
__device__ __forceinline__ bool spin_until(Smem& S, F cond) {
  if (cond()) return true;
  const long long t0 = clock64();
  while (!cond()) {
    if (failed(S)) return false;
    if (clock64() - t0 > kSpinCycles) {
      set_err(S, kTimeout);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

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
  if (j >= rem) return kWin;                  // literals reach the block end: last sequence
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

// ---------------------------------------------------------------------------
// parser warp
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ void parser_body(Smem& S, const Chunk& c, int p, uint32_t lane) {
  ParserSmem& P = S.ps[p];
  const uint8_t* win8 = reinterpret_cast<const uint8_t*>(P.winw);
  uint32_t tail = 0;
  // The compressed bytes of this parser's next segment are copied into shared
  // memory (16-byte cp.async, zero-filled past the block) while it parses the
  // current one.  Needs a 16-byte aligned block; otherwise bytes come from L1/L2.
  const bool pf = (reinterpret_cast<uintptr_t>(c.src) & 15) == 0;
  uint32_t pf_base[2] = {0xffffffffu, 0xffffffffu};
  auto prefetch = [&](int b, uint32_t j) {
    if (j >= c.n_seg) {
      pf_base[b] = 0xffffffffu;
    } else {
      const uint32_t base = c.seg_in(j) & ~15u;
      pf_base[b] = base;
      for (uint32_t q = lane; q < kInBuf / 16; q += 32) {
        const uint32_t o = base + 16 * q;
        const uint32_t nb = o < c.src_size ? min(16u, c.src_size - o) : 0u;
        cp_async16(&P.inbuf[b][16 * q], nb ? c.src + o : c.src, nb);
      }
    }
    cp_async_commit();
  };
  int cur = 0;
  if (pf) prefetch(0, p);
  for (uint32_t j = p; j < c.n_seg; j += kParsers, cur ^= 1) {
    if (pf) {
      prefetch(cur ^ 1, j + kParsers);
      cp_async_wait1();
      __syncwarp();
    }
    const uint8_t* buf = P.inbuf[cur];
    const uint32_t bbase = pf ? pf_base[cur] : 0xffffffffu;
    const uint32_t bend = pf ? min(bbase + kInBuf, c.src_size) : 0u;
    const uint32_t hi = c.seg_out(j + 1);
    uint32_t op = c.seg_out(j);
    uint32_t ip = c.seg_in(j);
    while (op < hi) {
      if (failed(S)) return;
      if (ip >= c.src_size) { set_err(S, ZMOE_CHUNK_INPUT_OVERRUN); return; }
      const uint32_t rem = c.src_size - ip;
      const uint32_t avail = rem < kStop ? rem : kStop;
      const uint8_t* win;
      if (pf && ip >= bbase && ip + avail <= bend && ip - bbase + kWin + 8 <= kInBuf) {
        win = buf + (ip - bbase);                  // window already in shared memory
      } else {
        // ---- stage [ip, ip + kWin) with aligned 32-bit loads --------------------
        const uintptr_t beg = reinterpret_cast<uintptr_t>(c.src);
        const uintptr_t end = beg + c.src_size;
        const uintptr_t addr = beg + ip;
        const uint32_t shift = (uint32_t)(addr & 3);
        for (uint32_t q = lane; q < kWin / 4 + 2; q += 32) {
          const uintptr_t wa = addr - shift + 4 * q;
          uint32_t v = 0;
          if (wa >= beg && wa + 4 <= end) {
            v = __ldg(reinterpret_cast<const uint32_t*>(wa));
          } else {
            for (uint32_t b = 0; b < 4; ++b)
              if (wa + b >= beg && wa + b < end)
                v |= (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(wa + b)) << (8 * b);
          }
          P.winw[q] = v;
        }
        __syncwarp();
        win = win8 + shift;
      }
      // ---- token starts: next-token table in registers, pointer doubling ----------
      // Lane l owns window positions 8l..8l+7; table entries are bytes
      // (255 = the chain stops), packed 4 per register, fetched with shuffles.
      uint32_t jt[kLevels][2];
      {
        const uintptr_t wa = reinterpret_cast<uintptr_t>(win) + 8 * lane;
        const uint32_t* aw = reinterpret_cast<const uint32_t*>(wa & ~uintptr_t(3));
        const uint32_t sh = (uint32_t)(wa & 3) * 8;
        const uint32_t w0 = aw[0], w1 = aw[1], w2 = aw[2];
        const uint32_t b03 = __funnelshift_r(w0, w1, sh), b47 = __funnelshift_r(w1, w2, sh);
        uint32_t r0 = 0, r1 = 0;
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
          const uint32_t i = 8 * lane + q;
          const uint32_t t = ((q < 4 ? b03 : b47) >> (8 * (q & 3))) & 0xFFu;
          uint32_t nx = kStop;
          if (i < avail) {
            const uint32_t ll = t >> 4;
            if (ll == 15 || (t & 15) == 15) {
              nx = next_token(win, i, avail, rem);           // length extensions: slow path
            } else {
              const uint32_t j = i + 1 + ll;
              if (j < rem && j + 2 <= avail) nx = j + 2;
            }
            if (nx > kStop) nx = kStop;
          }
          if (q < 4) r0 |= nx << (8 * q); else r1 |= nx << (8 * (q - 4));
        }
        jt[0][0] = r0;
        jt[0][1] = r1;
      }
#pragma unroll
      for (int k = 0; k + 1 < kLevels; ++k) {
        uint32_t r0 = 0, r1 = 0;
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
          const uint32_t v = ((q < 4 ? jt[k][0] : jt[k][1]) >> (8 * (q & 3))) & 0xFFu;
          const int src = (int)(v >> 3);
          const uint32_t a = __shfl_sync(kFull, jt[k][0], src), b = __shfl_sync(kFull, jt[k][1], src);
          const uint32_t e = v & 7;
          uint32_t nv = ((e < 4 ? a : b) >> (8 * (e & 3))) & 0xFFu;
          if (v == kStop) nv = kStop;
          if (q < 4) r0 |= nv << (8 * q); else r1 |= nv << (8 * (q - 4));
        }
        jt[k + 1][0] = r0;
        jt[k + 1][1] = r1;
      }
      uint32_t pp = 0;
#pragma unroll
      for (int k = 0; k < kLevels; ++k) {
        const int src = (int)(pp >> 3);
        const uint32_t a = __shfl_sync(kFull, jt[k][0], src), b = __shfl_sync(kFull, jt[k][1], src);
        const uint32_t e = pp & 7;
        const uint32_t nv = ((e < 4 ? a : b) >> (8 * (e & 3))) & 0xFFu;
        if (((lane >> k) & 1) && pp != kStop) pp = nv;
      }
      bool valid = pp < avail;
      auto byte_at = [&](uint32_t pos) -> uint32_t {
        const uint32_t rel = pos - ip;
        if (rel < avail) return win[rel];
        if (pos >= bbase && pos < bend) return buf[pos - bbase];
        return __ldg(c.src + pos);
      };
      // ---- sequence header of this lane --------------------------------------------
      uint32_t ll = 0, ml = 0, off = 0, lit_pos = 0, seq_end = 0;
      int lerr = 0;
      if (valid) {
        const uint32_t tok = win[pp];
        uint32_t q = ip + pp + 1;
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
      const uint64_t len = valid ? (uint64_t)ll + ml : 0;
      uint64_t incl = len;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const uint64_t v = __shfl_up_sync(kFull, incl, d);
        if (lane >= (uint32_t)d) incl += v;
      }
      const uint64_t ostart = (uint64_t)op + incl - len;
      valid = valid && ostart < hi;
      const uint64_t oend = min(ostart + len, (uint64_t)hi);
      const unsigned fit = __ballot_sync(kFull, valid && oend - op <= kBatch);
      const int cnt = __popc(__ballot_sync(kFull, valid));
      int nb = fit == kFull ? 32 : __ffs(~fit) - 1;
      nb = min(nb, cnt);
      const bool long_mode = nb == 0;
      const int used = long_mode ? 1 : nb;
      const bool mine = (int)lane < used;
      const uint64_t ms = ostart + ll;
      if (mine && !lerr && ml > 0 && ms < oend && (off == 0 || off > ms)) lerr = ZMOE_CHUNK_BAD_OFFSET;
      const unsigned emask = __ballot_sync(kFull, mine && lerr != 0);
      if (emask) { set_err(S, __shfl_sync(kFull, lerr, __ffs(emask) - 1)); return; }
      const uint32_t be = (uint32_t)__shfl_sync(kFull, oend, used - 1);
      if (be == op) { set_err(S, ZMOE_CHUNK_SHORT_OUTPUT); return; }   // empty final sequence

      // ---- wait for a free slot --------------------------------------------------
      if (!spin_until(S, [&] { return tail - vload(&S.q_head[p]) < (uint32_t)kSlots; })) return;
      Slot& sl = P.slot[tail % kSlots];
      if (!long_mode) {
        // One descriptor per output byte, spread over the lanes by position.
        // The owner sequence of byte r is found from a bitmap of sequence
        // starts (warp OR-reductions), its fields by shuffles.
        const uint32_t n = be - op;
        const uint32_t srel = mine ? (uint32_t)(ostart - op) : 0xffffffffu;
        const uint32_t mrel = (uint32_t)(ms - op);
        uint32_t startw[kBatch / 32], before[kBatch / 32];
        uint32_t acc = 0;
#pragma unroll
        for (uint32_t w = 0; w < kBatch / 32; ++w) {
          const uint32_t bit = (srel >> 5) == w ? (1u << (srel & 31)) : 0u;
          startw[w] = __reduce_or_sync(kFull, bit);
          before[w] = acc;
          acc += __popc(startw[w]);
        }
        const uint32_t lane_mask = (2u << lane) - 1u;   // bits 0..lane
        bool internal = false;
#pragma unroll
        for (uint32_t w = 0; w < kBatch / 32; ++w) {
          if (w * 32 >= n) break;                         // uniform
          const uint32_t r = lane + 32 * w;
          int own = (int)(before[w] + __popc(startw[w] & lane_mask)) - 1;
          own = max(0, min(own, used - 1));
          const uint32_t o_s = __shfl_sync(kFull, srel, own);
          const uint32_t o_m = __shfl_sync(kFull, mrel, own);
          const uint32_t o_lit = __shfl_sync(kFull, lit_pos, own);
          const uint32_t o_off = __shfl_sync(kFull, off, own);
          if (r < n) {
            uint32_t d;
            if (r < o_m) {
              d = kLit | byte_at(o_lit + (r - o_s));
            } else {
              const uint32_t k = r - o_m;
              uint32_t kk = k;
              if (o_off <= k) kk = k % o_off;
              const uint32_t s = op + o_m - o_off + kk;   // o_off <= ms: checked above
              if (s >= op) { d = kInternal | (s - op); internal = true; }
              else d = s;
            }
            sl.desc[r] = d;
          }
        }
        // sources produced inside the batch: chase them to a literal or an
        // earlier batch (rare; skipped when no lane has one)
        if (__any_sync(kFull, internal)) {
          __syncwarp();
          for (uint32_t r = lane; r < n; r += 32) {
            uint32_t d = *(volatile uint32_t*)&sl.desc[r];
            uint32_t steps = 0;
            while ((d & kInternal) && steps++ < kBatch) d = *(volatile uint32_t*)&sl.desc[d & ~kInternal];
            if (d & kInternal) { set_err(S, kTimeout); break; }
            *(volatile uint32_t*)&sl.desc[r] = d;
          }
        }
        if (lane == 0) { sl.mode = 0; }
      } else if (lane == 0) {
        sl.mode = 1;
        sl.l_ll = (uint32_t)min((uint64_t)ll, (uint64_t)(be - op));
        sl.l_lit = lit_pos;
        sl.l_ml = be - op - sl.l_ll;
        sl.l_off = off;
      }
      if (lane == 0) {
        sl.bs = op;
        sl.n = be - op;
      }
      __threadfence_block();
      __syncwarp();
      ++tail;
      if (lane == 0) vstore(&S.q_tail[p], tail);
      ip = __shfl_sync(kFull, seq_end, used - 1);
      op = be;
      if (op < hi && ip >= c.src_size) { set_err(S, ZMOE_CHUNK_SHORT_OUTPUT); return; }
    }
  }
}

// Every exit waits for the parser's own asynchronous copies into shared memory.
__device__ void parser(Smem& S, const Chunk& c, int p, uint32_t lane) {
  parser_body(S, c, p, lane);
  cp_async_wait0();
  __syncwarp();
}

// ---------------------------------------------------------------------------
// resolver warp
// ---------------------------------------------------------------------------
__device__ void resolver(Smem& S, const Chunk& c, uint32_t lane) {
  uint32_t head[kParsers] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < c.n_seg; ++j) {
    const int q = j % kParsers;
    const uint32_t hi = c.seg_out(j + 1);
    uint32_t pos = c.seg_out(j);
    while (pos < hi) {
      if (!spin_until(S, [&] { return vload(&S.q_tail[q]) != head[q]; })) return;
      __threadfence_block();
      Slot& sl = S.ps[q].slot[head[q] % kSlots];
      const uint32_t bs = sl.bs, n = sl.n, mode = sl.mode;
      if (bs != pos || n == 0) { set_err(S, kTimeout); return; }
      if (mode == 0) {
        if (!spin_until(S, [&] { return vload(&S.flush_pos) + kRing >= bs + n; })) return;
        uint32_t v[kBatch / 32];
#pragma unroll
        for (uint32_t i = 0; i < kBatch / 32; ++i) {
          const uint32_t r = lane + 32 * i;
          if (r < n) {
            const uint32_t d = sl.desc[r];
            v[i] = (d & kLit) ? (d & 0xFFu) : (uint32_t)S.ring[c.ri(d)];
          }
        }
        __syncwarp();
#pragma unroll
        for (uint32_t i = 0; i < kBatch / 32; ++i) {
          const uint32_t r = lane + 32 * i;
          if (r < n) S.ring[c.ri(bs + r)] = (uint8_t)v[i];
        }
      } else {
        // A long sequence can exceed the window: publish progress every 1 KiB so
        // the flusher keeps draining while the resolver writes.
        const uint32_t ll = sl.l_ll, lit = sl.l_lit, ml = sl.l_ml, o = sl.l_off;
        auto publish = [&](uint32_t upto) {
          __threadfence_block();
          __syncwarp();
          if (lane == 0) vstore(&S.res_pos, upto);
        };
        for (uint32_t k0 = 0; k0 < ll; k0 += 32) {
          const uint32_t e = bs + k0 + 32;
          if (!spin_until(S, [&] { return vload(&S.flush_pos) + kRing >= e; })) return;
          const uint32_t k = k0 + lane;
          if (k < ll) S.ring[c.ri(bs + k)] = __ldg(c.src + lit + k);
          __syncwarp();
          if (((k0 + 32) & 1023) == 0) publish(bs + k0 + 32);
        }
        const uint32_t m0 = bs + ll;
        for (uint32_t k0 = 0; k0 < ml; k0 += 32) {
          const uint32_t e = m0 + k0 + 32;
          if (!spin_until(S, [&] { return vload(&S.flush_pos) + kRing >= e; })) return;
          const uint32_t k = k0 + lane;
          uint32_t v = 0;
          if (k < ml) {
            const uint32_t m = lane / o + 1;      // most recent equal byte before this step
            v = S.ring[c.ri(m0 + k - o * m)];
          }
          __syncwarp();
          if (k < ml) S.ring[c.ri(m0 + k)] = (uint8_t)v;
          __syncwarp();
          if (((k0 + 32) & 1023) == 0 && k0 + 32 < ml) publish(m0 + k0 + 32);
        }
      }
      __threadfence_block();
      __syncwarp();
      ++head[q];
      if (lane == 0) {
        vstore(&S.res_pos, bs + n);
        vstore(&S.q_head[q], head[q]);
      }
      pos = bs + n;
    }
  }
}

// ---------------------------------------------------------------------------
// flusher warp
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack2(uint32_t e4, uint32_t s4, uint32_t sel) {
  const uint32_t e2 = __byte_perm(e4, 0, sel);
  const uint32_t s2 = __byte_perm(s4, 0, sel);
  return ((s2 & 0x00800080u) << 8) | (e2 << 7) | (s2 & 0x007F007Fu);
}

__device__ void flusher(Smem& S, const Chunk& c, uint32_t lane) {
  const uint32_t N = c.out_size;
  // vector path when the sign+mantissa plane and the output reach 16-byte
  // boundaries at the same element
  const uintptr_t sa = reinterpret_cast<uintptr_t>(c.sm), da = reinterpret_cast<uintptr_t>(c.dst);
  const uint32_t head = (uint32_t)((16 - (sa & 15)) & 15);
  const bool vec = ((da + 2 * (uintptr_t)head) & 15) == 0;
  uint32_t e = 0;
  while (e < N) {
    uint32_t avail = 0;
    if (!spin_until(S, [&] { avail = vload(&S.res_pos); return avail > e; })) return;
    __threadfence_block();
    uint32_t stop = avail;
    if (vec) {
      // scalar up to the first aligned element, then 16 elements per lane
      const uint32_t h = min(max(head, e), avail);
      for (uint32_t i = e + lane; i < h; i += 32)
        c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
      uint32_t v0 = h;
      const uint32_t units = (avail - v0) / 16;
      constexpr int kUnroll = 8;                // sign+mantissa loads in flight per lane
      for (uint32_t u0 = 0; u0 < units; u0 += 32 * kUnroll) {
        uint4 sv[kUnroll];
#pragma unroll
        for (int q = 0; q < kUnroll; ++q) {
          const uint32_t u = u0 + lane + 32 * q;
          if (u < units) sv[q] = __ldg(reinterpret_cast<const uint4*>(c.sm + v0 + 16 * u));
        }
#pragma unroll
        for (int q = 0; q < kUnroll; ++q) {
          const uint32_t u = u0 + lane + 32 * q;
          if (u >= units) break;
          const uint32_t i = v0 + 16 * u;
          const uint4 ev = *reinterpret_cast<const uint4*>(&S.ring[c.ri(i)]);
          uint4 lo, hi;
          lo.x = pack2(ev.x, sv[q].x, 0x4140); lo.y = pack2(ev.x, sv[q].x, 0x4342);
          lo.z = pack2(ev.y, sv[q].y, 0x4140); lo.w = pack2(ev.y, sv[q].y, 0x4342);
          hi.x = pack2(ev.z, sv[q].z, 0x4140); hi.y = pack2(ev.z, sv[q].z, 0x4342);
          hi.z = pack2(ev.w, sv[q].w, 0x4140); hi.w = pack2(ev.w, sv[q].w, 0x4342);
          uint4* o = reinterpret_cast<uint4*>(c.dst + i);
          o[0] = lo;
          o[1] = hi;
        }
      }
      stop = v0 + 16 * units;
      if (avail == N) {                         // block done: flush the tail too
        for (uint32_t i = stop + lane; i < N; i += 32)
          c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
        stop = N;
      }
      if (stop <= e) {                          // nothing aligned yet: wait for more
        if (!spin_until(S, [&] { return vload(&S.res_pos) >= min(N, e + 16 + head); })) return;
        continue;
      }
    } else {
      for (uint32_t i = e + lane; i < avail; i += 32)
        c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
    }
    __syncwarp();
    e = stop;
    if (lane == 0) vstore(&S.flush_pos, e);
  }
}

__global__ void __launch_bounds__(kWarps * 32)
decode_kernel(const zmoe_chunk* __restrict__ chunks, int n_chunks, int32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const zmoe_chunk d = chunks[blockIdx.x];
  Chunk c;
  c.src = d.src;
  c.sm = d.sm;
  c.dst = d.dst;
  c.index = (d.index && d.n_index > 0) ? d.index : nullptr;
  c.src_size = d.src_size;
  c.out_size = d.out_size;
  c.n_seg = c.index ? d.n_index : 1;
  {
    const uint32_t head = (uint32_t)((16 - (reinterpret_cast<uintptr_t>(d.sm) & 15)) & 15);
    c.rofs = (16 - head) & 15;
  }
  if (threadIdx.x == 0) {
    S.err = (!c.src || !c.sm || !c.dst || c.src_size == 0) ? ZMOE_CHUNK_BAD_DESC : 0;
    S.res_pos = 0;
    S.flush_pos = 0;
    for (int p = 0; p < kParsers; ++p) { S.q_tail[p] = 0; S.q_head[p] = 0; }
  }
  __syncthreads();
  if (!S.err && c.out_size > 0) {
    if (warp < kParsers) parser(S, c, warp, lane);
    else if (warp == kResolver) resolver(S, c, lane);
    else flusher(S, c, lane);
  }
  __syncthreads();
  if (threadIdx.x == 0) status[blockIdx.x] = S.err;
}

}  // namespace

zmoe_status launch_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status, cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  const int smem = (int)sizeof(Smem);
  ZMOE_CUDA_RET(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  decode_kernel<<<n_chunks, kWarps * 32, smem, stream>>>(chunks, n_chunks, status);
  return launch_status("decode_kernel");
}

}  // namespace zmoe
