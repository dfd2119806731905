// Fused LZ4-block decode + plane recombine (sm_100a).
//
// Reference path replaced: per exponent chunk, LZ4_decompress_safe_partial
// on a CPU worker (csrc/tensor_engine/compressors.cpp:195-211, driven by
// tensor_engine.cpp:421-474), a memcpy into a pinned dock, then the recombine
// kernel (csrc/kernels/tensor_recover.cu:12-43) reading both planes over
// zero-copy host memory.
//
// LZ4HC matches chain back through earlier matches (median offset ~20 KB), so
// the bytes of a block depend on each other almost serially; the token stream
// does not.  One CTA of 6 warps decodes one block in two overlapped stages:
//
//  * Source map (4 parser warps).  A slice index built when the block is
//    loaded (zmoe_lz4_build_index) names, for every 256 output bytes, the
//    sequence that contains that byte.  Each lane parses one 256-byte slice on
//    its own (a parser warp covers an 8 KiB window) and writes one 32-bit
//    entry per output byte into a map ring in L2-resident scratch: a literal
//    value, or the position of a byte with the same value.  For a match byte
//    the position is the most recent equal byte before the 2 KiB step that
//    holds it (for a run of period o, the latest earlier copy), so it is
//    always inside the 64 KiB window; a source inside the step itself is
//    recorded in a shared-memory list and chased through the map once the
//    window is mapped.  No entry depends on its own step.
//  * Resolve (1 resolver warp + 1 flusher warp).  The map entries of the next
//    2 KiB step are copied into shared memory (cp.async) while the resolver
//    gathers the current step's bytes from a 64 KiB shared-memory window of
//    decoded exponents and writes them back into the window.  The flusher
//    follows, merging 16 exponent bytes
//    with 16 sign+mantissa bytes (128-bit loads) into BF16 (two 128-bit
//    stores per lane); the resolver never overwrites a byte the flusher has
//    not consumed.
//
// A chunk without an index (zmoe_chunk.index == NULL) is decoded by warp 0
// alone in one pass straight into the output (no scratch needed).
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
constexpr uint32_t kSlice = 256;              // output bytes parsed by one lane
constexpr uint32_t kWindow = 32 * kSlice;     // output bytes mapped by one parser pass
constexpr uint32_t kStep = 2048;              // output bytes resolved per resolver step
constexpr uint32_t kRing = 65536;             // decoded-exponent window
constexpr uint32_t kRingMask = kRing - 1;
constexpr uint32_t kMapEntries = ZMOE_MAP_ENTRIES;   // source-map ring per chunk (scratch)
constexpr uint32_t kMapMask = kMapEntries - 1;
static_assert(kSlice == ZMOE_SLICE_BYTES, "slice index granularity");
constexpr uint32_t kMapWindows = kMapEntries / kWindow;
constexpr uint32_t kLit = 0x80000000u;        // map entry: literal value in bits 0..7
constexpr uint32_t kInner = 0x40000000u;      // map entry (parse time only): source inside its step
constexpr long long kSpinCycles = 2000000000LL;   // ~1 s at 1.9 GHz
constexpr unsigned kFull = 0xffffffffu;
constexpr int32_t kTimeout = 5;

static_assert((kMapEntries & (kMapEntries - 1)) == 0 && kMapWindows >= 2, "map ring");

constexpr uint32_t kChaseCap = 256;           // in-step sources recorded per parser window

struct Smem {
  uint8_t ring[kRing];
  __align__(16) uint32_t mbuf[2][kStep];      // resolver: map entries of the current/next step
  uint32_t chase[kParsers][kChaseCap];        // positions whose source lies inside their step
  uint32_t n_chase[kParsers];
  uint32_t win_ready[kMapWindows];            // window w mapped: win_ready[w % n] == w + 1
  uint32_t res_pos;                           // bytes [0, res_pos) resolved into the ring
  uint32_t res_win;                           // windows fully resolved (map slots reusable)
  uint32_t flush_pos;                         // bytes [0, flush_pos) consumed by the flusher
  int32_t err;
};

struct Chunk {
  const uint8_t* src;
  const uint8_t* sm;
  uint16_t* dst;
  const uint32_t* index;
  uint32_t* map;
  uint32_t src_size, out_size, n_index;
  uint32_t rofs;   // ring index of position i is (i + rofs) & kRingMask; makes 16-byte
                   // groups that the flusher loads aligned both in the ring and in memory
  __device__ __forceinline__ uint32_t ri(uint32_t pos) const { return (pos + rofs) & kRingMask; }
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
    __nanosleep(64);
  }
  return true;
}

// One LZ4 sequence header at ip: literal count and position, match offset and
// length, position of the next token.  Returns 0 or a ZMOE_CHUNK_* error.
struct Seq {
  uint32_t ll, lit, off, ml, next;
  bool last;
};

__device__ __forceinline__ int read_seq(const uint8_t* __restrict__ src, uint32_t size, uint32_t ip, Seq& s) {
  if (ip >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
  const uint32_t tok = __ldg(src + ip);
  uint32_t q = ip + 1;
  uint32_t ll = tok >> 4;
  if (ll == 15) {
    uint32_t b;
    do {
      if (q >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
      b = __ldg(src + q++);
      ll += b;
    } while (b == 255 && ll < (1u << 30));
  }
  if ((uint64_t)q + ll > size) return ZMOE_CHUNK_INPUT_OVERRUN;
  s.ll = ll;
  s.lit = q;
  q += ll;
  s.off = 0;
  s.ml = 0;
  s.last = q == size;
  if (!s.last) {
    if (q + 2 > size) return ZMOE_CHUNK_INPUT_OVERRUN;
    s.off = __ldg(src + q) | ((uint32_t)__ldg(src + q + 1) << 8);
    q += 2;
    uint32_t ml = tok & 15;
    if (ml == 15) {
      uint32_t b;
      do {
        if (q >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
        b = __ldg(src + q++);
        ml += b;
      } while (b == 255 && ml < (1u << 30));
    }
    s.ml = ml + 4;
  }
  s.next = q;
  return 0;
}

// ---------------------------------------------------------------------------
// parser warps: source map
// ---------------------------------------------------------------------------
__device__ void parser(Smem& S, const Chunk& c, int p, uint32_t lane) {
  const uint32_t n_win = (c.out_size + kWindow - 1) / kWindow;
  for (uint32_t w = p; w < n_win; w += kParsers) {
    // the map slots of window w are free once window w - kMapWindows is resolved
    if (w >= kMapWindows && !spin_until(S, [&] { return vload(&S.res_win) > w - kMapWindows; })) return;
    const uint32_t g = w * 32 + lane;                 // slice of this lane
    const uint32_t b0 = g * kSlice;
    const uint32_t b1 = min(b0 + kSlice, c.out_size);
    int err = 0;
    bool overflow = false;
    if (b0 < c.out_size) {
      if (g >= c.n_index) {
        err = ZMOE_CHUNK_BAD_DESC;
      } else {
        uint32_t ip = __ldg(c.index + 2 * g);
        uint32_t so = __ldg(c.index + 2 * g + 1);     // output start of the sequence at ip
        uint32_t e = b0;
        uint32_t r0 = 0, r1 = 0, r2 = 0;              // entries waiting for a 128-bit store
        auto put = [&](uint32_t pos, uint32_t v) {
          switch (pos & 3) {
            case 0: r0 = v; break;
            case 1: r1 = v; break;
            case 2: r2 = v; break;
            default: reinterpret_cast<uint4*>(c.map)[(pos & kMapMask) >> 2] = make_uint4(r0, r1, r2, v);
          }
        };
        auto note_inner = [&](uint32_t pos) {         // chase this position after the window
          const uint32_t slot = atomicAdd(&S.n_chase[p], 1u);
          if (slot < kChaseCap) S.chase[p][slot] = pos; else overflow = true;
        };
        if (so > b0) err = ZMOE_CHUNK_BAD_DESC;
        while (!err && e < b1) {
          Seq s;
          err = read_seq(c.src, c.src_size, ip, s);
          if (err) break;
          const uint32_t ms = so + s.ll;              // first match byte
          const uint32_t me = ms + s.ml;
          const uint32_t o = s.off;
          if (s.ml > 0 && (o == 0 || o > ms)) { err = ZMOE_CHUNK_BAD_OFFSET; break; }
          // literals
          for (; e < b1 && e < ms; ++e) put(e, kLit | __ldg(c.src + s.lit + (e - so)));
          // match bytes: a byte with the same value before the 2 KiB step of e
          for (; e < b1 && e < me; ++e) {
            const uint32_t step0 = e & ~(kStep - 1);
            const uint32_t k = e - ms;
            uint32_t v;
            if (k < o) {                              // plain copy: the source itself
              v = e - o;
            } else {                                  // overlapping copy of period o
              const uint32_t base = ms - o + k % o;  // first copy, in [ms - o, ms)
              v = base < step0 ? base + o * ((step0 - 1 - base) / o) : base;   // latest below the step
            }
            if (v >= step0) {                         // inside the step: chase after the window
              note_inner(e);
              v |= kInner;
            }
            put(e, v);
          }
          if (e < b1) {
            if (s.last) { err = ZMOE_CHUNK_SHORT_OUTPUT; break; }
            ip = s.next;
            so = me;
          }
        }
        if (!err && (e & 3)) {                        // partial group at the chunk end
          const uint32_t i0 = e & ~3u;
          c.map[i0 & kMapMask] = r0;
          if (e - i0 > 1) c.map[(i0 + 1) & kMapMask] = r1;
          if (e - i0 > 2) c.map[(i0 + 2) & kMapMask] = r2;
        }
      }
    }
    const unsigned emask = __ballot_sync(kFull, err != 0);
    if (emask) {
      set_err(S, __shfl_sync(kFull, err, __ffs(emask) - 1));
      return;
    }
    // chase sources inside the same 2 KiB step through the map (written by any
    // lane of this warp) until a literal or a byte before the step
    __threadfence_block();
    __syncwarp();
    const uint32_t n_list = min(vload(&S.n_chase[p]), kChaseCap);
    const bool full_scan = __any_sync(kFull, overflow);
    auto chase_one = [&](uint32_t i) {
      uint32_t v = __ldcg(c.map + (i & kMapMask));
      if (!(v & kInner)) return;
      uint32_t steps = 0;
      while ((v & kInner) && steps++ < kStep) v = __ldcg(c.map + ((v & ~kInner) & kMapMask));
      if (v & kInner) { set_err(S, kTimeout); return; }
      c.map[i & kMapMask] = v;
    };
    if (!full_scan) {
      for (uint32_t q = lane; q < n_list; q += 32) chase_one(S.chase[p][q]);
    } else {
      for (uint32_t i = b0; i < b1; ++i) chase_one(i);
    }
    __syncwarp();
    if (lane == 0) vstore(&S.n_chase[p], 0);
    __threadfence_block();
    __syncwarp();
    if (lane == 0) vstore(&S.win_ready[w % kMapWindows], w + 1);
  }
}

// ---------------------------------------------------------------------------
// resolver warp
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Copy the map entries of step t (2048 x 4 bytes, contiguous in the ring) to mbuf[t & 1].
__device__ __forceinline__ void fetch_step(Smem& S, const Chunk& c, uint32_t t, uint32_t lane) {
  const uint32_t* src = c.map + ((t * kStep) & kMapMask);
  uint32_t* dst = S.mbuf[t & 1];
  for (uint32_t q = lane; q < kStep / 4; q += 32) cp_async16(dst + 4 * q, src + 4 * q);
  cp_async_commit();
}

__device__ void resolver_body(Smem& S, const Chunk& c, uint32_t lane) {
  const uint32_t n_steps = (c.out_size + kStep - 1) / kStep;
  constexpr uint32_t kStepsPerWin = kWindow / kStep;
  auto ready = [&](uint32_t t) {
    const uint32_t w = t / kStepsPerWin;
    return vload(&S.win_ready[w % kMapWindows]) == w + 1;
  };
  // map entries of step t + 1 are copied while step t resolves
  if (!spin_until(S, [&] { return ready(0); })) return;
  __threadfence_block();
  fetch_step(S, c, 0, lane);
  bool have_next = true;                              // a copy for step t is in flight
  for (uint32_t t = 0; t < n_steps; ++t) {
    const uint32_t s0 = t * kStep, s1 = min(s0 + kStep, c.out_size);
    if (!have_next) {
      if (!spin_until(S, [&] { return ready(t); })) return;
      __threadfence_block();
      fetch_step(S, c, t, lane);
    }
    have_next = false;
    if (t + 1 < n_steps && ready(t + 1)) {
      __threadfence_block();
      fetch_step(S, c, t + 1, lane);
      have_next = true;
      cp_async_wait1();
    } else {
      cp_async_wait0();
    }
    __syncwarp();
    if (!spin_until(S, [&] { return vload(&S.flush_pos) + kRing >= s1; })) return;
    // gather the whole step, then write it (a write may reuse the window slot
    // of a source read in this step)
    const uint32_t* mb = S.mbuf[t & 1];
    uint32_t val[kStep / 128];
#pragma unroll
    for (uint32_t i = 0; i < kStep / 128; ++i) {
      const uint32_t r = 128 * i + 4 * lane;
      const uint4 m = *reinterpret_cast<const uint4*>(mb + r);
      const uint32_t mv[4] = {m.x, m.y, m.z, m.w};
      uint32_t packed = 0;
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b) {
        const uint32_t d = mv[b];
        uint32_t x = d & 0xFFu;
        if (!(d & kLit) && s0 + r + b < s1) x = S.ring[c.ri(d)];
        packed |= x << (8 * b);
      }
      val[i] = packed;
    }
    __syncwarp();
#pragma unroll
    for (uint32_t i = 0; i < kStep / 128; ++i) {
      const uint32_t e = s0 + 128 * i + 4 * lane;
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b)
        if (e + b < s1) S.ring[c.ri(e + b)] = (uint8_t)(val[i] >> (8 * b));
    }
    __threadfence_block();
    __syncwarp();
    if (lane == 0) {
      vstore(&S.res_pos, s1);
      if (s1 == c.out_size || (s1 % kWindow) == 0) vstore(&S.res_win, (s1 + kWindow - 1) / kWindow);
    }
  }
}

// Every exit waits for the resolver's own asynchronous copies into shared memory.
__device__ void resolver(Smem& S, const Chunk& c, uint32_t lane) {
  resolver_body(S, c, lane);
  cp_async_wait0();
  __syncwarp();
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
      const uint32_t v0 = h;
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

// ---------------------------------------------------------------------------
// chunks without an index: one warp, straight into the output
// ---------------------------------------------------------------------------
// Lane 0 walks the tokens; the warp copies each sequence cooperatively.  A
// match byte k of a copy with offset o repeats the byte at (start - o + k mod o),
// so a copy needs no serial loop.  Sources are read back from the BF16 output
// (exponent = bits 7..14) through L2.
__device__ int decode_unindexed(const Chunk& c, uint32_t lane) {
  uint32_t ip = 0, op = 0;
  int err = 0;
  while (op < c.out_size) {
    Seq s;
    if (lane == 0) err = read_seq(c.src, c.src_size, ip, s);
    err = __shfl_sync(kFull, err, 0);
    if (err) return err;
    s.ll = __shfl_sync(kFull, s.ll, 0);
    s.lit = __shfl_sync(kFull, s.lit, 0);
    s.off = __shfl_sync(kFull, s.off, 0);
    s.ml = __shfl_sync(kFull, s.ml, 0);
    s.next = __shfl_sync(kFull, s.next, 0);
    s.last = __shfl_sync(kFull, (int)s.last, 0) != 0;
    const uint32_t lit_n = min(s.ll, c.out_size - op);
    for (uint32_t i = lane; i < lit_n; i += 32)
      c.dst[op + i] = (uint16_t)recombine(__ldg(c.sm + op + i), __ldg(c.src + s.lit + i));
    op += lit_n;
    if (op >= c.out_size) break;
    if (s.last) return ZMOE_CHUNK_SHORT_OUTPUT;
    if (s.off == 0 || s.off > op) return ZMOE_CHUNK_BAD_OFFSET;
    __threadfence_block();
    __syncwarp();
    const uint32_t mlen = min(s.ml, c.out_size - op);
    for (uint32_t k0 = 0; k0 < mlen; k0 += 32) {
      const uint32_t k = k0 + lane;
      // source: most recent copy before this 32-byte step (written already)
      uint32_t v = 0;
      if (k < mlen) {
        const uint32_t base = op - s.off + (k < s.off ? k : k % s.off);
        const uint32_t step0 = op + k0;
        const uint32_t src = base < step0 ? base + s.off * ((step0 - 1 - base) / s.off) : base;
        v = ((uint32_t)__ldcg(c.dst + src) >> 7) & 0xFFu;
      }
      __syncwarp();
      if (k < mlen) c.dst[op + k] = (uint16_t)recombine(__ldg(c.sm + op + k), v);
      __threadfence_block();
      __syncwarp();
    }
    op += mlen;
    ip = s.next;
  }
  return 0;
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
  c.map = d.map;
  c.src_size = d.src_size;
  c.out_size = d.out_size;
  c.n_index = d.n_index;
  {
    const uint32_t head = (uint32_t)((16 - (reinterpret_cast<uintptr_t>(d.sm) & 15)) & 15);
    c.rofs = (16 - head) & 15;
  }
  if (threadIdx.x == 0) {
    bool bad = !c.src || !c.sm || !c.dst || c.src_size == 0;
    if (c.index && (!c.map || (reinterpret_cast<uintptr_t>(c.map) & 15) || d.seg_bytes != kSlice)) bad = true;
    S.err = bad ? ZMOE_CHUNK_BAD_DESC : 0;
    S.res_pos = 0;
    S.res_win = 0;
    S.flush_pos = 0;
    for (uint32_t w = 0; w < kMapWindows; ++w) S.win_ready[w] = 0;
    for (int p = 0; p < kParsers; ++p) S.n_chase[p] = 0;
  }
  __syncthreads();
  if (!S.err && c.out_size > 0) {
    if (!c.index) {
      if (warp == 0) {
        const int e = decode_unindexed(c, lane);
        if (e && lane == 0) set_err(S, e);
      }
    } else if (warp < kParsers) {
      parser(S, c, warp, lane);
    } else if (warp == kResolver) {
      resolver(S, c, lane);
    } else {
      flusher(S, c, lane);
    }
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
