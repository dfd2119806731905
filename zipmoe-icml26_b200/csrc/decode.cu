// Fused LZ4-block decode + plane recombine (sm_100a).
//
// Reference path replaced: per exponent chunk, LZ4_decompress_safe_partial
// on a CPU worker (csrc/tensor_engine/compressors.cpp:195-211, driven by
// tensor_engine.cpp:421-474), a memcpy into a pinned dock, then the recombine
// kernel (csrc/kernels/tensor_recover.cu:12-43) reading both planes over
// zero-copy host memory.
//
// Exponent planes compress into many short sequences (about one per 7 output
// bytes, 92% of the bytes in matches, match chains tens deep), so the bytes of
// a block depend on each other almost serially while the token stream does
// not.  Output is handled in 64 KiB regions, by two kernels on one stream:
//
//  map_kernel, 16 CTAs of 256 threads per chunk, each mapping every 16th
//  region (every chunk at once), one region at a time:
//  1. Stage: the region's compressed bytes are copied into shared memory.
//  2. Map: a slice index built when the block is loaded (zmoe_lz4_build_index)
//     names, for every 256 output bytes, the sequence that contains the first
//     of them.  Each thread maps one slice on its own and writes one 32-bit
//     entry per output byte into the chunk's scratch: a literal value, or the
//     position of an earlier byte with the same value.  For a match byte that
//     position is the source itself, or, for a run longer than its offset,
//     the latest equal byte before the 2 KiB step holding it when one exists.
//  3. Chase: once the whole region is mapped, the 4-byte groups holding an
//     entry whose source lies inside its own step are listed, and the CTA's
//     threads share the list: each such entry is replaced by following the
//     step's entries back to a literal or to a byte before the step.  Each
//     region also gets a status word.
//
//  resolve_kernel, one CTA of 512 threads per chunk:
//  4. Resolve: step by step (2 KiB, 4 bytes per thread), the entries are
//     copied into shared memory (cp.async, three steps ahead) and every byte is
//     gathered from a 64 KiB shared-memory window of decoded exponents.  The
//     whole step is gathered before it is written.
//  5. Flush: each step first writes out the 2 KiB it is about to overwrite in
//     the window (decoded 32 steps earlier) as BF16, with sign+mantissa bytes
//     that came in with the step's entries; the last 64 KiB follow the last
//     step.
//
// Only the resolve is serial within a chunk; mapping every region at once
// keeps the SMs busy when few chunks are decoded.  A chunk without an index
// (zmoe_chunk.index == NULL) is decoded by warp 0 of its resolve CTA alone, in
// one pass straight into the output (no scratch needed).
//
// There are no inter-warp flags and no waits other than barriers and the
// completion of the CTA's own asynchronous copies.  Errors (bad offsets,
// lengths past the block, a block ending short of out_size, an index that
// does not match the block) set the chunk's status word; the kernels never
// trap.  Output past out_size is clipped (the targetOutputSize = out_size
// behaviour of LZ4_decompress_safe_partial).
#include "common.cuh"

namespace zmoe {
namespace {

constexpr int kThreads = 256;
constexpr uint32_t kSlice = 256;                    // output bytes parsed by one thread
constexpr uint32_t kRegion = kThreads * kSlice;     // output bytes per region (64 KiB)
constexpr uint32_t kStep = 2048;                    // output bytes resolved per step
constexpr int kRThreads = 512;                      // threads of a resolve CTA
constexpr uint32_t kPerThread = kStep / kRThreads;  // bytes resolved per thread and step
constexpr uint32_t kRing = 65536;                   // decoded-exponent window
constexpr uint32_t kRingMask = kRing - 1;
constexpr uint32_t kStage = 48 * 1024;              // staged compressed bytes per region
constexpr uint32_t kTGroups = 4;                    // groups per lane between transposed map stores
constexpr uint32_t kTPitch = kTGroups + 1;          // uint4 per lane in tbuf (padded: no bank conflicts)
constexpr uint32_t kMapBufs = 4;                    // map-entry buffers of the resolve
constexpr uint32_t kAhead = kMapBufs - 1;           // steps whose entries are in flight
constexpr uint32_t kLit = 0x80000000u;              // map entry: literal value in bits 0..7
constexpr uint32_t kInner = 0x40000000u;            // map entry: source inside its own step
constexpr uint32_t kPosMask = kInner - 1;
constexpr unsigned kFull = 0xffffffffu;

static_assert(kSlice == ZMOE_SLICE_BYTES, "slice index granularity");
static_assert(kRegion == ZMOE_MAP_ENTRIES, "one map entry per byte of a region");
static_assert(kRegion <= kRing, "a region's sources stay inside the window");
static_assert(kStep % kSlice == 0 && kRegion % kStep == 0, "slices nest in steps nest in regions");
static_assert(kPerThread == 4, "one 128-bit map load per thread and step");
static_assert((kTGroups * 16) % 32 == 0 && 32 % kTGroups == 0 && (kSlice / 4) % kTGroups == 0,
              "a lane's transposed groups fill whole 32-byte sectors");
static_assert((kRegion / 4) * sizeof(uint16_t) <= kStage && kRegion / 4 <= 65536, "the chase list fits the stage");

struct MapSmem {                                    // map_kernel
  uint8_t stage[kStage];                            // compressed bytes of the region, then the chase list
  uint4 tbuf[kThreads * kTPitch];                    // per warp: 32 lanes x kTPitch (map_slice_staged)
  uint32_t wsum[kThreads / 32];
  int32_t err;
};

struct Smem {                                       // resolve_kernel
  uint8_t ring[kRing];
  uint32_t mbuf[kMapBufs][kStep];                   // map entries of the next steps
  uint32_t sbuf[kMapBufs][kStep / 4];               // sign+mantissa words of the next steps' flush windows
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
                   // groups that the flush loads aligned both in the ring and in memory
  __device__ __forceinline__ uint32_t ri(uint32_t pos) const { return (pos + rofs) & kRingMask; }
};

template <class SM>
__device__ __forceinline__ void set_err(SM& S, int32_t code) { atomicCAS(&S.err, 0, code); }


__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One LZ4 sequence header at ip: literal count and position, match offset and
// length, position of the next token.  Returns 0 or a ZMOE_CHUNK_* error.
struct Seq {
  uint32_t ll, lit, off, ml, next;
  bool last;
};

template <class ByteAt>
__device__ __forceinline__ int read_seq(ByteAt byte_at, uint32_t size, uint32_t ip, Seq& s) {
  if (ip >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
  const uint32_t tok = byte_at(ip);
  uint32_t q = ip + 1;
  uint32_t ll = tok >> 4;
  if (ll == 15) {
    uint32_t b;
    do {
      if (q >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
      b = byte_at(q++);
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
    s.off = byte_at(q) | (byte_at(q + 1) << 8);
    q += 2;
    uint32_t ml = tok & 15;
    if (ml == 15) {
      uint32_t b;
      do {
        if (q >= size) return ZMOE_CHUNK_INPUT_OVERRUN;
        b = byte_at(q++);
        ml += b;
      } while (b == 255 && ml < (1u << 30));
    }
    s.ml = ml + 4;
  }
  s.next = q;
  return 0;
}

// ---------------------------------------------------------------------------
// phase 1: stage the compressed bytes of region r
// ---------------------------------------------------------------------------
// The region's sequences start in [index[g0].in, index[g0 + 256].in]; the last
// one's header and literals may run past that, so a margin is staged too and
// anything beyond the staged range is read from global memory.
struct StageRange {
  uint32_t lo, len;   // compressed bytes [lo, lo + len) are in S.u.stage
};

__device__ __forceinline__ StageRange stage_range(const Chunk& c, uint32_t r) {
  StageRange st{0, 0};
  const uint32_t g0 = r * kThreads;
  if (g0 >= c.n_index) return st;
  const uint32_t in_lo = __ldg(c.index + 2 * g0);
  const uint32_t in_hi = g0 + kThreads < c.n_index ? __ldg(c.index + 2 * (g0 + kThreads)) : c.src_size;
  const uint32_t lo = in_lo & ~15u;
  if (lo >= c.src_size) return st;
  const uint32_t full = (c.src_size - lo) & ~15u;                 // whole 16-byte units inside the block
  const uint32_t want = (uint32_t)min((uint64_t)in_hi + 256 - lo, (uint64_t)kStage);
  st.lo = lo;
  st.len = min(full, (want + 15) & ~15u);
  return st;
}

__device__ __forceinline__ void stage_issue(uint8_t* stage, const Chunk& c, const StageRange& st) {
  for (uint32_t q = 16 * threadIdx.x; q < st.len; q += 16 * kThreads) cp_async16(stage + q, c.src + st.lo + q);
  cp_async_commit();
}

// ---------------------------------------------------------------------------
// phase 2: map one 256-byte slice per thread
// ---------------------------------------------------------------------------
// The sequence being mapped: output bytes [so, ms) are literals (compressed
// byte lit_base + position), [ms, me) match bytes.
struct Run {
  uint32_t ms, me, o, lit_base, next;
  bool last;
  bool periodic;                                      // the match is longer than its offset
};

template <class ByteAt>
__device__ __forceinline__ int open_run(ByteAt byte_at, uint32_t size, uint32_t ip, uint32_t so, Run& r) {
  Seq s;
  const int err = read_seq(byte_at, size, ip, s);
  if (err) return err;
  r.ms = so + s.ll;
  r.me = r.ms + s.ml;
  r.o = s.off;
  if (s.ml > 0 && (r.o == 0 || r.o > r.ms)) return ZMOE_CHUNK_BAD_OFFSET;
  r.lit_base = s.lit - so;
  r.next = s.next;
  r.last = s.last;
  r.periodic = s.ml > r.o;
  return 0;
}

// Source of match byte p (p >= ms) of a copy with offset o.  A plain copy
// (p - ms < o, all but 0.01% of the bytes of an exponent plane) reads byte
// p - o.  A byte of a run longer than its offset repeats every o bytes back to
// ms - o; with wrap = max(ms, step0) its source is the copy in [wrap - o, wrap):
// below the step when the run began before it, else the run's first copy.
// Either way a source at or after step0 lies inside the step and is marked
// for the chase.
__device__ __forceinline__ uint32_t periodic_source(uint32_t p, uint32_t ms, uint32_t o, uint32_t step0) {
  const uint32_t wrap = max(ms, step0);
  return wrap - o + (p - wrap) % o;
}
// Match entries hold the source position plus the chunk's ring offset rofs,
// so the resolve's ring index is the entry's low 16 bits.
__device__ __forceinline__ uint32_t match_entry(uint32_t p, uint32_t ms, uint32_t o, bool periodic, uint32_t step0,
                                                uint32_t rofs) {
  uint32_t v = p - o;
  if (periodic && p - ms >= o) v = periodic_source(p, ms, o, step0);
  return (v + rofs) | (v >= step0 ? kInner : 0u);
}

// The slice is walked in 64 groups of 4 bytes, the same count in every lane.
// A sequence that starts inside (or right after) a group is opened before the
// group's entries are formed (every sequence but the last covers at least 4
// bytes, so a group meets at most two), each byte takes its fields from the
// sequence it belongs to, and the group is one 128-bit map store.  Lanes
// diverge only while a header is parsed.
//
// Staged walk: a header is read from the staged bytes only when the header
// and its literals lie wholly inside them (one range check per sequence);
// otherwise the walk stops with miss set and the slice is mapped again by the
// checked walk.  The block's last sequence (no match part) always misses, as
// the stage holds whole 16-byte units only.
struct FastRun {
  uint32_t ms, me, o, lit_t, pe, next;   // literal p is stage[p + lit_t]; p >= pe: periodic byte
};

// Opens the sequence whose token is at compressed position ip and whose
// output starts at so.  Returns false if any of its header or literal bytes
// is outside the stage; a bad offset sets err and leaves r as it was.
__device__ __forceinline__ bool fast_open(const uint8_t* stage, uint32_t lo, uint32_t len, uint32_t ip, uint32_t so,
                                          FastRun& r, int& err) {
  uint32_t q = ip - lo;
  if (q >= len) return false;
  const uint32_t tok = stage[q++];
  uint32_t ll = tok >> 4;
  if (ll == 15) {
    uint32_t b;
    do {
      if (q >= len) return false;
      b = stage[q++];
      ll += b;
    } while (b == 255);
  }
  const uint32_t lit = q;                              // ll < 255 * len: no overflow below
  if (q + ll + 2 > len) return false;
  q += ll;
  const uint32_t o = stage[q] | ((uint32_t)stage[q + 1] << 8);
  q += 2;
  uint32_t ml = tok & 15;
  if (ml == 15) {
    uint32_t b;
    do {
      if (q >= len) return false;
      b = stage[q++];
      ml += b;
    } while (b == 255);
  }
  ml += 4;
  const uint32_t ms = so + ll;
  if (o == 0 || o > ms) {                              // r keeps its fields: a dead lane reads them
    err = ZMOE_CHUNK_BAD_OFFSET;
    return true;
  }
  r.ms = ms;
  r.me = ms + ml;
  r.o = o;
  r.lit_t = lit - so;
  r.pe = ml > o ? r.ms + o : 0xFFFFFFFFu;
  r.next = lo + q;
  return true;
}

// Every lane of the warp runs the staged walk for the same 64 groups (a lane
// with no slice to map, or one that met an error or a miss, goes on as a dead
// lane whose entries are discarded), so that the warp can store its entries
// through a transpose: each lane puts kTGroups = 4 groups (64 bytes of its
// slice) into tbuf, then each store instruction writes 8 runs of 64 bytes (two
// whole 32-byte sectors each), 4 lanes per run, instead of 32 lanes each
// writing 16 bytes into a different line.
// tbuf: this warp's 32 x kTPitch uint4.
__device__ int map_slice_staged(const uint8_t* stage, uint4* tbuf, const Chunk& c, const StageRange& st, uint32_t g,
                                bool active, bool& miss, uint64_t& inner) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t b0 = g * kSlice;
  const uint32_t b1 = min(b0 + kSlice, c.out_size);
  const uint32_t step0 = b0 & ~(kStep - 1);            // a slice lies inside one step
  int err = 0;
  bool dead = !active;
  FastRun cur{0u, 0u, 1u, 0u, 0xFFFFFFFFu, 0u};        // a dead lane's fields: match bytes, stage index 0
  if (!dead) {
    const uint2 ix = __ldg(reinterpret_cast<const uint2*>(c.index) + g);
    const uint32_t so = ix.y;                          // output start of the sequence at ix.x
    if (so > b0) {
      err = ZMOE_CHUNK_BAD_DESC;
      dead = true;
    } else if (!fast_open(stage, st.lo, st.len, ix.x, so, cur, err)) {
      miss = true;
      dead = true;
    } else if (err || cur.me <= b0) {                  // cur.me <= b0: the index names a sequence ending before b0
      if (!err) err = ZMOE_CHUNK_BAD_DESC;
      dead = true;
    }
  }
  // c.map: the region's entries; this warp's 32 slices start at slice g - lane
  uint4* wmap = reinterpret_cast<uint4*>(c.map) + (size_t)(threadIdx.x - lane) * (kSlice / 4);
  FastRun nxt = cur;                                   // read only for bytes at or past cur.me
  for (uint32_t k = 0; k < kSlice / 4; ++k) {
    const uint32_t p0 = b0 + 4 * k;
    // a live lane has cur.me > p0 here, and an opened sequence covers at least 4 bytes
    const bool turn = !dead && cur.me <= p0 + 4 && cur.me < b1;
    if (turn) {
      if (!fast_open(stage, st.lo, st.len, cur.next, cur.me, nxt, err)) {
        miss = true;
        dead = true;
      } else if (err) {
        dead = true;
      }
    }
    uint32_t x[4];
#pragma unroll
    for (uint32_t b = 0; b < 4; ++b) {
      const uint32_t p = p0 + b;
      const bool in_a = p < cur.me;
      const uint32_t ms = in_a ? cur.ms : nxt.ms, lit_t = in_a ? cur.lit_t : nxt.lit_t;
      const uint32_t o = in_a ? cur.o : nxt.o, pe = in_a ? cur.pe : nxt.pe;
      const bool lit = p < ms;
      const uint32_t lb = stage[lit ? p + lit_t : 0u];
      uint32_t v = p - o;
      if (p >= pe) v = periodic_source(p, ms, o, step0);
      v = (v + c.rofs) | (v >= step0 ? kInner : 0u);
      x[b] = lit ? (kLit | lb) : v;
    }
    tbuf[lane * kTPitch + k % kTGroups] = make_uint4(x[0], x[1], x[2], x[3]);
    if (!dead && p0 < b1 && ((x[0] | x[1] | x[2] | x[3]) & kInner)) inner |= 1ull << k;
    if (turn && !dead) cur = nxt;
    if (k % kTGroups == kTGroups - 1) {
      __syncwarp();
      const uint32_t piece = lane % kTGroups, k0 = k + 1 - kTGroups;
#pragma unroll
      for (uint32_t it = 0; it < kTGroups; ++it) {
        const uint32_t src = it * (32 / kTGroups) + lane / kTGroups;   // lane whose line this lane writes
        wmap[src * (kSlice / 4) + k0 + piece] = tbuf[src * kTPitch + piece];
      }
      __syncwarp();
    }
  }
  return dead ? err : 0;
}

// Checked walk: every compressed byte is read from the stage when it lies
// there and from global memory otherwise, with every bound checked.
__device__ int map_slice_checked(const uint8_t* stage, const Chunk& c, const StageRange& st, uint32_t g,
                                 uint64_t& inner) {
  const uint32_t b0 = g * kSlice;
  const uint2 ix = __ldg(reinterpret_cast<const uint2*>(c.index) + g);
  const uint32_t so = ix.y;                            // output start of the sequence at ix.x
  if (so > b0) return ZMOE_CHUNK_BAD_DESC;
  const uint32_t b1 = min(b0 + kSlice, c.out_size);
  const uint32_t step0 = b0 & ~(kStep - 1);            // a slice lies inside one step
  auto checked = [&](uint32_t q) -> uint32_t {
    const uint32_t d = q - st.lo;
    return d < st.len ? (uint32_t)stage[d] : (uint32_t)__ldg(c.src + q);
  };
  auto entry = [&](uint32_t p, const Run& a, const Run& b) -> uint32_t {
    const Run& r = p < a.me ? a : b;
    if (p < r.ms) return kLit | checked(r.lit_base + p);
    return match_entry(p, r.ms, r.o, r.periodic, step0, c.rofs);
  };
  Run cur;
  int err = open_run(checked, c.src_size, ix.x, so, cur);
  if (err) return err;
  if (cur.me <= b0) return ZMOE_CHUNK_BAD_DESC;        // the index names a sequence ending before b0
  uint4* map4 = reinterpret_cast<uint4*>(c.map);
  Run nxt = cur;                                       // read only for bytes at or past cur.me
  for (uint32_t p0 = b0; p0 < b1; p0 += 4) {
    const bool turn = cur.me <= p0 + 4 && cur.me < b1;
    if (turn) {
      if (cur.last) return ZMOE_CHUNK_SHORT_OUTPUT;
      if ((err = open_run(checked, c.src_size, cur.next, cur.me, nxt)) != 0) return err;
      if (nxt.me < min(p0 + 4, b1)) return ZMOE_CHUNK_SHORT_OUTPUT;   // only the last one can be this short
    }
    const uint4 x = make_uint4(entry(p0 + 0, cur, nxt), entry(p0 + 1, cur, nxt), entry(p0 + 2, cur, nxt),
                               entry(p0 + 3, cur, nxt));
    map4[(p0 % kRegion) / 4] = x;
    if ((x.x | x.y | x.z | x.w) & kInner) inner |= 1ull << ((p0 - b0) / 4);
    if (turn) cur = nxt;
  }
  return 0;
}

// inner: bit k set when group k (bytes 4k..4k+3 of the slice) holds an entry
// whose source lies inside its own step.
// Called by every thread of the CTA (the staged walk stores warp-wide).
__device__ int map_slice(const uint8_t* stage, uint4* tbuf, const Chunk& c, const StageRange& st, uint32_t g,
                         uint64_t& inner) {
  inner = 0;
  const bool have = g * kSlice < c.out_size;
  const bool valid = have && g < c.n_index;
  bool miss = false;
  int err = 0;
  if (st.len != 0) {                                   // the same in every thread of the CTA
    err = map_slice_staged(stage, tbuf, c, st, g, valid, miss, inner);
    if (!miss && valid) return err;
    inner = 0;
  }
  if (!have) return 0;
  if (!valid) return ZMOE_CHUNK_BAD_DESC;
  return map_slice_checked(stage, c, st, g, inner);   // some byte was not staged: checked reads
}

// ---------------------------------------------------------------------------
// phase 3: chase the entries whose source lies inside their own step
// ---------------------------------------------------------------------------
// Once every slice of the region is mapped, each entry whose source lies
// inside its own step is replaced by the entry of that source, followed back
// to a literal or to a position before the step; the resolve then gathers each
// step with no chase.  Other threads rewrite entries of the step at the same
// time; whichever value a read sees (marked or final) names the same byte
// value.  Positions strictly decrease along a chase, so it ends within a
// step's length; a chase that leaves the step or does not move back is an
// index/block mismatch.
//
// The groups to chase are gathered into one list for the CTA, so that a slice
// with many of them (a long run of short copies) is shared by all threads
// instead of holding the region's barrier for one thread.  Each thread takes
// two groups at a time and follows their eight entries in lockstep, one hop
// (an L2 load) per round for every entry still marked.
constexpr uint32_t kChaseGroups = 2;

__device__ int chase_groups(const Chunk& c, uint32_t rbase, const uint16_t* list, uint32_t total) {
  uint4* map4 = reinterpret_cast<uint4*>(c.map);
  int err = 0;
  for (uint32_t i0 = threadIdx.x; i0 < total; i0 += kThreads * kChaseGroups) {
    uint32_t gi[kChaseGroups], x[4 * kChaseGroups], cur[4 * kChaseGroups];
    bool live[kChaseGroups];
#pragma unroll
    for (uint32_t k = 0; k < kChaseGroups; ++k) {
      const uint32_t i = i0 + k * kThreads;
      live[k] = i < total;
      gi[k] = live[k] ? list[i] : 0u;
    }
#pragma unroll
    for (uint32_t k = 0; k < kChaseGroups; ++k) {
      const uint4 v = live[k] ? __ldcg(map4 + gi[k]) : make_uint4(kLit, kLit, kLit, kLit);
      x[4 * k + 0] = v.x; x[4 * k + 1] = v.y; x[4 * k + 2] = v.z; x[4 * k + 3] = v.w;
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b) {
        cur[4 * k + b] = rbase + 4 * gi[k] + b;
        if (cur[4 * k + b] >= c.out_size) x[4 * k + b] &= ~kInner;   // padding of the last group: never read
      }
    }
    for (;;) {
      bool any = false;
#pragma unroll
      for (uint32_t q = 0; q < 4 * kChaseGroups; ++q) {
        if (x[q] & kInner) {
          const uint32_t src = (x[q] & kPosMask) - c.rofs;
          const uint32_t step0 = cur[q] & ~(kStep - 1);
          if (src >= cur[q] || src < step0) {
            err = ZMOE_CHUNK_BAD_DESC;
            x[q] = kLit;
          } else {
            cur[q] = src;
            x[q] = __ldcg(c.map + (src - rbase));
            any = true;
          }
        }
      }
      if (!any) break;
    }
#pragma unroll
    for (uint32_t k = 0; k < kChaseGroups; ++k)
      if (live[k]) __stcg(map4 + gi[k], make_uint4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]));
  }
  return err;
}

// Exclusive prefix sum of v over the CTA; total gets the sum.  wsum: kThreads / 32 words.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* wsum, uint32_t& total) {
  const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (uint32_t d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(kFull, inc, d);
    if (lane >= d) inc += y;
  }
  if (lane == 31) wsum[w] = inc;
  __syncthreads();
  uint32_t before = 0;
  total = 0;
#pragma unroll
  for (uint32_t k = 0; k < kThreads / 32; ++k) {
    const uint32_t t = wsum[k];
    before += k < w ? t : 0u;
    total += t;
  }
  return before + inc - v;
}

__device__ void flush_range(Smem& S, const Chunk& c, uint32_t f0, uint32_t f1, uint32_t head, bool vec);

// ---------------------------------------------------------------------------
// phase 4: resolve the region's steps through the shared-memory window
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack2(uint32_t e4, uint32_t s4, uint32_t sel);

// Resolves steps [0, n_steps) of the chunk.  Thread q copies (cp.async) map
// entries 4q..4q+3 of every step; warp v resolves bytes 128v..128v+127, lane
// l the bytes l, l + 32, l + 64 and l + 96 of those.
//
// The output is written as it leaves the ring: step t overwrites the slots of
// positions 64 KiB before it, so from step kLag = 32 on, each step first
// writes BF16 for its flush window, positions
// [(t - kLag) * kStep + head, + kStep): thread q takes 4 of them, whose
// sign+mantissa word came in with the step's entries (cp.async, 4 bytes,
// aligned because sm + head is).  The window's lowest positions were written
// by the previous step's window, and its highest are overwritten only by the
// next step.  Positions [0, head) go out at step kLag, and whatever no window
// covered (the whole chunk when it has at most kLag steps) after the last
// step.
__device__ int resolve_steps(Smem& S, const Chunk& c, uint32_t head, bool vec, bool vec8) {
  constexpr uint32_t kLag = kRegion / kStep;
  const uint32_t R1 = c.out_size;
  const uint32_t n_steps = (R1 + kStep - 1) / kStep;
  const uint32_t q = threadIdx.x;
  const uint32_t j0 = kPerThread * q;
  int err = 0;
  // map entries (and window words) run kAhead steps ahead of the resolve (one
  // commit group per step, empty past the end, so wait_group counts stay uniform)
  const uint32_t* fsrc = c.map + j0;                   // this thread's entries of the next step to fetch
  uint32_t* mrow = &S.mbuf[0][j0];                     // its entries in buffer 0; buffer k is k * kStep further
  auto fetch = [&](uint32_t tf) {
    cp_async16(mrow + (tf % kMapBufs) * kStep, fsrc);
    if (tf >= kLag) cp_async4(&S.sbuf[tf % kMapBufs][q], c.sm + (tf - kLag) * kStep + head + j0);
  };
  for (uint32_t p = 0; p < kAhead; ++p) {
    if (p < n_steps) fetch(p);
    cp_async_commit();
    fsrc += kStep;
  }
  const uint32_t jb = 128 * (q / 32) + (q % 32);      // this thread's first byte of a step
  uint32_t w = (jb + c.rofs) & kRingMask;              // its ring index
  for (uint32_t t = 0; t < n_steps; ++t) {
    const uint32_t s0 = t * kStep;
    // buffer (t + kAhead) % kMapBufs last held step t - 1, which this thread has read
    if (t + kAhead < n_steps) fetch(t + kAhead);
    fsrc += kStep;
    cp_async_commit();
    cp_async_wait<kAhead>();
    __syncthreads();                                   // A: the step's entries landed; the previous steps' bytes visible
    // this thread's bytes: positions s0 + jb + 32k, k = 0..3 (a warp takes 128
    // consecutive bytes, so one gather instruction reads a few runs of
    // consecutive sources instead of 32 scattered ones)
    const uint32_t* mb = S.mbuf[t % kMapBufs] + jb;
    uint32_t x[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) x[k] = mb[32 * k];
    const bool tail = s0 + kStep > R1;                 // the chunk's last step (the same in every thread)
    if (tail) {
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k)
        if (s0 + jb + 32 * k >= R1) x[k] = kLit;       // past the chunk end: entry never written
    }
    // map_kernel left every entry a literal or a position before the step
    if ((x[0] | x[1] | x[2] | x[3]) & kInner) {
      err = ZMOE_CHUNK_BAD_DESC;
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k) x[k] = kLit;
    }
    uint32_t val[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) val[k] = (x[k] & kLit) ? (x[k] & 0xFFu) : (uint32_t)S.ring[x[k] & kRingMask];
    if (t >= kLag) {                                   // the flush window, before its slots are overwritten
      const uint32_t i = (t - kLag) * kStep + head + j0;
      const uint32_t ev = *reinterpret_cast<const uint32_t*>(&S.ring[c.ri(i)]);
      const uint32_t sv = S.sbuf[t % kMapBufs][q];
      const uint32_t lo = pack2(ev, sv, 0x4140), hi = pack2(ev, sv, 0x4342);
      if (vec8) {
        __stcs(reinterpret_cast<uint2*>(c.dst + i), make_uint2(lo, hi));
      } else {
        c.dst[i] = (uint16_t)lo;
        c.dst[i + 1] = (uint16_t)(lo >> 16);
        c.dst[i + 2] = (uint16_t)hi;
        c.dst[i + 3] = (uint16_t)(hi >> 16);
      }
      if (t == kLag && q < head) c.dst[q] = (uint16_t)recombine(__ldg(c.sm + q), S.ring[c.ri(q)]);
    }
    __syncthreads();                                   // B: the whole step is gathered, the window read
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k)
      if (!tail || s0 + jb + 32 * k < R1) S.ring[(w + 32 * k) & kRingMask] = (uint8_t)val[k];
    w = (w + kStep) & kRingMask;
  }
  cp_async_wait<0>();
  __syncthreads();                                     // the last step's bytes visible
  const uint32_t f0 = n_steps > kLag ? (n_steps - kLag) * kStep + head : 0u;
  flush_range(S, c, min(f0, R1), R1, head, vec);
  return err;
}

// ---------------------------------------------------------------------------
// phase 5: BF16 out
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack2(uint32_t e4, uint32_t s4, uint32_t sel) {
  const uint32_t e2 = __byte_perm(e4, 0, sel);
  const uint32_t s2 = __byte_perm(s4, 0, sel);
  return ((s2 & 0x00800080u) << 8) | (e2 << 7) | (s2 & 0x007F007Fu);
}

// Writes positions [f0, f1).  vec: 16-element groups starting at head + 16u are
// 16-byte aligned in the sign+mantissa plane, the output and the ring.
__device__ void flush_range(Smem& S, const Chunk& c, uint32_t f0, uint32_t f1, uint32_t head, bool vec) {
  if (!vec) {
    for (uint32_t i = f0 + threadIdx.x; i < f1; i += kRThreads)
      c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
    return;
  }
  // first aligned group start >= f0, last aligned end <= f1
  const uint32_t v0 = f0 <= head ? head : head + ((f0 - head + 15) & ~15u);
  const uint32_t v1 = f1 <= head ? head : head + ((f1 - head) & ~15u);
  if (v0 >= v1) {
    for (uint32_t i = f0 + threadIdx.x; i < f1; i += kRThreads)
      c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
    return;
  }
  for (uint32_t i = f0 + threadIdx.x; i < v0; i += kRThreads)
    c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
  for (uint32_t i = v1 + threadIdx.x; i < f1; i += kRThreads)
    c.dst[i] = (uint16_t)recombine(__ldg(c.sm + i), S.ring[c.ri(i)]);
  const uint32_t units = (v1 - v0) / 16;
  constexpr int kUnroll = 4;                           // sign+mantissa loads in flight per thread
  for (uint32_t u0 = 0; u0 < units; u0 += kRThreads * kUnroll) {
    uint4 sv[kUnroll];
#pragma unroll
    for (int q = 0; q < kUnroll; ++q) {
      const uint32_t u = u0 + threadIdx.x + kRThreads * q;
      if (u < units) sv[q] = __ldcs(reinterpret_cast<const uint4*>(c.sm + v0 + 16 * u));
    }
#pragma unroll
    for (int q = 0; q < kUnroll; ++q) {
      const uint32_t u = u0 + threadIdx.x + kRThreads * q;
      if (u >= units) break;
      const uint32_t i = v0 + 16 * u;
      const uint4 ev = *reinterpret_cast<const uint4*>(&S.ring[c.ri(i)]);
      uint4 lo, hi;
      lo.x = pack2(ev.x, sv[q].x, 0x4140); lo.y = pack2(ev.x, sv[q].x, 0x4342);
      lo.z = pack2(ev.y, sv[q].y, 0x4140); lo.w = pack2(ev.y, sv[q].y, 0x4342);
      hi.x = pack2(ev.z, sv[q].z, 0x4140); hi.y = pack2(ev.z, sv[q].z, 0x4342);
      hi.z = pack2(ev.w, sv[q].w, 0x4140); hi.w = pack2(ev.w, sv[q].w, 0x4342);
      uint4* o = reinterpret_cast<uint4*>(c.dst + i);
      __stcs(o, lo);                                   // streaming: keep L2 for the map scratch
      __stcs(o + 1, hi);
    }
  }
}

// Status word of each region, after the map entries of the chunk's regions.
__device__ __forceinline__ int32_t* region_status(uint32_t* map, uint32_t n_reg) {
  return reinterpret_cast<int32_t*>(map + (size_t)n_reg * kRegion);
}

__device__ void resolve_chunk(Smem& S, const Chunk& c) {
  const uintptr_t sa = reinterpret_cast<uintptr_t>(c.sm), da = reinterpret_cast<uintptr_t>(c.dst);
  const uint32_t head = (uint32_t)((16 - (sa & 15)) & 15);
  const bool vec = ((da + 2 * (uintptr_t)head) & 15) == 0;
  const bool vec8 = ((da + 2 * (uintptr_t)head) & 7) == 0;
  const uint32_t n_reg = (c.out_size + kRegion - 1) / kRegion;
  const int32_t* rstat = region_status(c.map, n_reg);
  for (uint32_t r = 0; r < n_reg; ++r) {               // map_kernel's verdicts (the same in every thread)
    const int32_t mapped = __ldcg(rstat + r);
    if (mapped != 0) {
      if (threadIdx.x == 0) set_err(S, mapped);
      return;
    }
  }
  const int err = resolve_steps(S, c, head, vec, vec8);
  if (err) set_err(S, err);
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
  auto byte_at = [&](uint32_t q) -> uint32_t { return __ldg(c.src + q); };
  while (op < c.out_size) {
    Seq s;
    if (lane == 0) err = read_seq(byte_at, c.src_size, ip, s);
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

// Descriptor checks shared by both kernels.
__device__ __forceinline__ bool bad_desc(const zmoe_chunk& d) {
  bool bad = !d.src || !d.sm || !d.dst || d.src_size == 0 || d.out_size >= kInner;
  if (d.index && d.n_index > 0 &&
      (!d.map || (reinterpret_cast<uintptr_t>(d.map) & 15) || (reinterpret_cast<uintptr_t>(d.index) & 7) ||
       d.seg_bytes != kSlice))
    bad = true;
  return bad;
}

__device__ __forceinline__ Chunk chunk_of(const zmoe_chunk& d) {
  Chunk c;
  c.src = d.src;
  c.sm = d.sm;
  c.dst = d.dst;
  c.index = (d.index && d.n_index > 0) ? d.index : nullptr;
  c.map = d.map;
  c.src_size = d.src_size;
  c.out_size = d.out_size;
  c.n_index = d.n_index;
  const uint32_t head = (uint32_t)((16 - (reinterpret_cast<uintptr_t>(d.sm) & 15)) & 15);
  c.rofs = (16 - head) & 15;
  return c;
}

// Map and chase (phases 1-3) of the regions r = blockIdx.x, r + gridDim.x, ... of chunk
// blockIdx.y.  Every region's status word is written (0 or the first error),
// so the scratch needs no clearing between launches.
__global__ void __launch_bounds__(kThreads, 2)
map_kernel(const zmoe_chunk* __restrict__ chunks) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  MapSmem& M = *reinterpret_cast<MapSmem*>(smem_raw);
  const zmoe_chunk d = chunks[blockIdx.y];
  if (bad_desc(d) || !d.index || d.n_index == 0 || d.out_size == 0) return;   // resolve_kernel reports it
  const Chunk c = chunk_of(d);
  const uint32_t n_reg = (c.out_size + kRegion - 1) / kRegion;
  int32_t* rstat = region_status(d.map, n_reg);
  const bool src_aligned = (reinterpret_cast<uintptr_t>(c.src) & 15) == 0;
  for (uint32_t r = blockIdx.x; r < n_reg; r += gridDim.x) {
    const StageRange st = src_aligned ? stage_range(c, r) : StageRange{0, 0};
    if (threadIdx.x == 0) M.err = 0;
    stage_issue(M.stage, c, st);
    cp_async_wait<0>();
    __syncthreads();                                   // staged bytes and the cleared error visible
    Chunk cr = c;
    cr.map = d.map + (size_t)r * kRegion;
    const uint32_t g = r * kThreads + threadIdx.x;
    uint64_t inner;
    int err = map_slice(M.stage, M.tbuf + (threadIdx.x / 32) * 32 * kTPitch, cr, st, g, inner);
    if (err) inner = 0;
    // list the groups to chase (group index within the region), in the stage
    uint32_t total;
    uint32_t at = block_scan((uint32_t)__popcll(inner), M.wsum, total);   // its barrier: the stage is free
    uint16_t* list = reinterpret_cast<uint16_t*>(M.stage);
    while (inner) {
      list[at++] = (uint16_t)(threadIdx.x * (kSlice / 4) + (uint32_t)__ffsll((long long)inner) - 1);
      inner &= inner - 1;
    }
    __syncthreads();                                   // the list and every entry of the region written
    const int cerr = chase_groups(cr, r * kRegion, list, total);
    if (!err) err = cerr;
    if (err) set_err(M, err);
    __syncthreads();
    if (threadIdx.x == 0) rstat[r] = M.err;
    __syncthreads();                                   // before the stage and the error word are reused
  }
}

// Resolve and flush (phases 4-5) of chunk blockIdx.x after map_kernel, or the
// whole decode of a chunk without an index.
__global__ void __launch_bounds__(kRThreads, 2)
resolve_kernel(const zmoe_chunk* __restrict__ chunks, int32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>(smem_raw);
  const zmoe_chunk d = chunks[blockIdx.x];
  const bool bad = bad_desc(d);
  const Chunk c = chunk_of(d);
  if (threadIdx.x == 0) S.err = bad ? ZMOE_CHUNK_BAD_DESC : 0;
  __syncthreads();
  if (!bad && c.out_size > 0) {
    if (!c.index) {
      if ((threadIdx.x >> 5) == 0) {
        const int e = decode_unindexed(c, threadIdx.x & 31);
        if (e && threadIdx.x == 0) set_err(S, e);
      }
    } else {
      resolve_chunk(S, c);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) status[blockIdx.x] = S.err;
}

}  // namespace

zmoe_status launch_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status, cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  ZMOE_CHECK_ARG(n_chunks <= 65535, "decode_chunks: %d chunks in one launch (at most 65535)", n_chunks);
  constexpr int kMapColumns = 16;                     // map CTAs per chunk (each loops over regions)
  const int msmem = (int)sizeof(MapSmem), rsmem = (int)sizeof(Smem);
  static uint64_t attr_set = 0;                        // devices whose kernel attributes are set
  int dev = 0;
  ZMOE_CUDA_RET(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << (dev & 63)))) {
    ZMOE_CUDA_RET(cudaFuncSetAttribute(map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, msmem));
    ZMOE_CUDA_RET(cudaFuncSetAttribute(resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rsmem));
    attr_set |= 1ull << (dev & 63);
  }
  map_kernel<<<dim3(kMapColumns, n_chunks), kThreads, msmem, stream>>>(chunks);
  zmoe_status st = launch_status("map_kernel");
  if (st != ZMOE_OK) return st;
  resolve_kernel<<<n_chunks, kRThreads, rsmem, stream>>>(chunks, status);
  return launch_status("resolve_kernel");
}

}  // namespace zmoe

extern "C" uint64_t zmoe_decode_scratch_bytes(uint32_t out_size) {
  const uint64_t n_reg = ((uint64_t)out_size + zmoe::kRegion - 1) / zmoe::kRegion;
  return n_reg * zmoe::kRegion * 4 + (n_reg * 4 + 15) / 16 * 16;
}
