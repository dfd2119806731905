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
// Three launches per call, all chunks at once:
//  1. chain_kernel, one warp per chunk: the hash chains.  prev[i] is the
//     latest position j < i whose 4 bytes hash like those at i (15-bit
//     multiplicative hash), or kNone.  The warp walks the chunk 32 positions
//     at a time; lanes with equal hashes are found with __match_any_sync, so
//     the chains stay in position order exactly as a serial insertion makes
//     them.  The head of each bucket sits in shared memory.
//  2. match_kernel, one thread per position: the longest match among at most
//     max_attempts chain candidates inside the 64 KiB window (the first
//     candidate found wins ties, i.e. the nearest).  A match may not reach
//     into the block's last 5 bytes, and none starts in its last 12 (the LZ4
//     end-of-block rules).
//  3. emit_kernel, one warp per chunk: a greedy parse with one step of lazy
//     evaluation (a match is put off by one byte when the next position has a
//     longer one), and the block's bytes: token, literal-length bytes,
//     literals, little-endian offset, match-length bytes, then the last
//     literals.  A block that would not fit dst_capacity gets size 0.
//
// No launch waits on another thread or block, so nothing can hang; every
// index is bounded by the chunk's size.
#include "common.cuh"

namespace zmoe {
namespace {

constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr int kHashLog = 15;
constexpr uint32_t kHashSize = 1u << kHashLog;
constexpr uint32_t kMinMatch = 4;
constexpr uint32_t kLastLiterals = 5;                // the last 5 bytes are literals
constexpr uint32_t kMfLimit = 12;                    // no match starts in the last 12 bytes
constexpr uint32_t kMaxOffset = 65535;
constexpr unsigned kFull = 0xffffffffu;

struct EncChunk {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t* prev;                                    // scratch: [src_size] chain links
  uint32_t* mlen;                                    // scratch: [src_size] best match length (0: none)
  uint16_t* moff;                                    // scratch: [src_size] its offset
  uint32_t src_size, dst_capacity;
};

__device__ __forceinline__ uint32_t read4(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ uint32_t hash4(uint32_t v) { return (v * 2654435761u) >> (32 - kHashLog); }

__device__ __forceinline__ EncChunk enc_chunk_of(const zmoe_enc_chunk& d) {
  EncChunk c;
  c.src = d.src;
  c.dst = d.dst;
  const uint64_t n = d.src_size;
  uint8_t* base = reinterpret_cast<uint8_t*>(d.scratch);
  c.prev = reinterpret_cast<uint32_t*>(base);
  c.mlen = reinterpret_cast<uint32_t*>(base + 4 * n);
  c.moff = reinterpret_cast<uint16_t*>(base + 8 * n);
  c.src_size = d.src_size;
  c.dst_capacity = d.dst_capacity;
  return c;
}

// Positions are 32-bit with headroom: chunks above 1 GiB are refused.  An
// empty chunk needs neither source nor scratch.
__device__ __forceinline__ bool bad_enc(const zmoe_enc_chunk& d) {
  return !d.dst || (d.src_size && (!d.src || !d.scratch)) || (reinterpret_cast<uintptr_t>(d.scratch) & 15) != 0 ||
         d.src_size > (1u << 30);
}

// ---------------------------------------------------------------------------
// 1. hash chains (one warp per chunk)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32) chain_kernel(const zmoe_enc_chunk* __restrict__ chunks) {
  extern __shared__ uint32_t head[];                 // [kHashSize] latest position per bucket
  const zmoe_enc_chunk d = chunks[blockIdx.x];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  const uint32_t lane = threadIdx.x;
  for (uint32_t h = lane; h < kHashSize; h += 32) head[h] = kNone;
  __syncwarp();
  const uint32_t n = c.src_size;
  const uint32_t lt = lane == 0 ? 0u : (kFull >> (32 - lane));   // lanes below this one
  for (uint32_t i0 = 0; i0 < n; i0 += 32) {
    const uint32_t i = i0 + lane;
    const bool keyed = i + kMinMatch <= n;           // has 4 bytes to hash
    const uint32_t h = keyed ? hash4(read4(c.src + i)) : kHashSize + lane;   // unkeyed lanes match no one
    const uint32_t peers = __match_any_sync(kFull, h);
    const uint32_t below = peers & lt;
    uint32_t link = kNone;
    if (keyed) link = below ? i0 + (31 - __clz(below)) : head[h];
    __syncwarp();                                    // every read of head before the writes
    if (keyed && (peers >> lane) == 1u) head[h] = i; // the highest lane of its bucket
    if (i < n) c.prev[i] = link;
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// 2. longest match per position (one thread per position)
// ---------------------------------------------------------------------------
// A candidate's length is searched up to kLenCap bytes, so that long runs
// cost O(kLenCap) per position; the parse extends a capped match it keeps.
constexpr uint32_t kLenCap = 1024;

__global__ void __launch_bounds__(256) match_kernel(const zmoe_enc_chunk* __restrict__ chunks, int max_attempts) {
  const zmoe_enc_chunk d = chunks[blockIdx.y];
  if (bad_enc(d)) return;
  const EncChunk c = enc_chunk_of(d);
  const uint32_t n = c.src_size;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t best = 0, best_off = 0;
    if (i + kMfLimit <= n) {                          // a match may start here
      const uint32_t max_len = min(n - kLastLiterals - i, kLenCap);
      const uint32_t key = read4(c.src + i);
      uint32_t cand = c.prev[i];
      for (int a = 0; a < max_attempts && cand != kNone; ++a) {
        if (cand >= i || i - cand > kMaxOffset) break;   // links go strictly back; farther ones are out of the window
        if (read4(c.src + cand) == key) {
          uint32_t len = kMinMatch;
          while (len < max_len && c.src[cand + len] == c.src[i + len]) ++len;
          if (len > best) {
            best = len;
            best_off = i - cand;
            if (len >= max_len) break;
          }
        }
        cand = c.prev[cand];
      }
    }
    c.mlen[i] = best >= kMinMatch ? best : 0u;
    c.moff[i] = (uint16_t)best_off;
  }
}

// ---------------------------------------------------------------------------
// 3. parse and write the block (one warp per chunk)
// ---------------------------------------------------------------------------
// Bytes of the 255-run that follows a length nibble of 15 (rest = length - 15).
__device__ __forceinline__ uint32_t run_bytes(uint32_t rest) { return rest / 255 + 1; }

// rest as a 255-run at dst, the lanes striding over its bytes.
__device__ __forceinline__ void put_run(uint8_t* dst, uint32_t rest, uint32_t lane) {
  const uint32_t nb = rest / 255;
  for (uint32_t k = lane; k <= nb; k += 32) dst[k] = k < nb ? (uint8_t)255 : (uint8_t)(rest - nb * 255);
}

// One sequence at dst + op: token, literal-length run, literals, little-endian
// offset, match-length run; ml == 0 is the block's last literals (no match
// part).  Returns its size, or clears ok and writes nothing when it would pass
// cap.  Every argument is the same in all lanes.
__device__ uint32_t put_sequence(uint8_t* dst, uint32_t op, uint32_t cap, const uint8_t* lit, uint32_t ll,
                                 uint32_t off, uint32_t ml, uint32_t lane, bool& ok) {
  const uint32_t mcode = ml ? ml - kMinMatch : 0u;
  const uint32_t llb = ll >= 15 ? run_bytes(ll - 15) : 0u;
  const uint32_t mlb = ml && mcode >= 15 ? run_bytes(mcode - 15) : 0u;
  const uint32_t size = 1 + llb + ll + (ml ? 2 + mlb : 0u);
  if ((uint64_t)op + size > cap) {
    ok = false;
    return 0;
  }
  uint8_t* q = dst + op;
  if (lane == 0) q[0] = (uint8_t)(((ll >= 15 ? 15u : ll) << 4) | (ml ? (mcode >= 15 ? 15u : mcode) : 0u));
  if (llb) put_run(q + 1, ll - 15, lane);
  q += 1 + llb;
  for (uint32_t k = lane; k < ll; k += 32) q[k] = lit[k];
  if (ml) {
    q += ll;
    if (lane == 0) {
      q[0] = (uint8_t)(off & 0xFF);
      q[1] = (uint8_t)(off >> 8);
    }
    if (mlb) put_run(q + 2, mcode - 15, lane);
  }
  return size;
}

// The parse visits positions in order; a window of 32 is tested at once and
// the first position the serial parse would take is found with a ballot: a
// match of at least 4 whose successor (if it may start a match) is not longer.
__global__ void __launch_bounds__(32) emit_kernel(const zmoe_enc_chunk* __restrict__ chunks,
                                                  uint32_t* __restrict__ out_sizes) {
  const zmoe_enc_chunk d = chunks[blockIdx.x];
  const uint32_t lane = threadIdx.x;
  if (bad_enc(d)) {
    if (lane == 0) out_sizes[blockIdx.x] = 0;
    return;
  }
  const EncChunk c = enc_chunk_of(d);
  const uint32_t n = c.src_size;
  uint32_t i = 0, anchor = 0, op = 0;
  bool ok = true;
  while (ok && i + kMfLimit <= n) {
    const uint32_t j = i + lane;
    uint32_t len = 0;
    bool take = false;
    if (j + kMfLimit <= n) {
      len = c.mlen[j];
      if (len >= kMinMatch) take = !(j + 1 + kMfLimit <= n && c.mlen[j + 1] > len);   // lazy: the next is longer
    }
    const uint32_t taken = __ballot_sync(kFull, take);
    if (!taken) {
      i += 32;
      continue;
    }
    const uint32_t f = __ffs(taken) - 1;
    uint32_t ml = __shfl_sync(kFull, len, f);
    i += f;
    const uint32_t off = c.moff[i];
    if (ml == kLenCap) {                             // capped in the search: extend it here
      const uint32_t end = n - kLastLiterals;
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
    op += put_sequence(c.dst, op, c.dst_capacity, c.src + anchor, i - anchor, off, ml, lane, ok);
    i += ml;
    anchor = i;
  }
  if (ok) op += put_sequence(c.dst, op, c.dst_capacity, c.src + anchor, n - anchor, 0, 0, lane, ok);
  if (lane == 0) out_sizes[blockIdx.x] = ok ? op : 0u;
}

}  // namespace

zmoe_status launch_encode_chunks(const zmoe_enc_chunk* chunks, int n_chunks, int max_attempts, uint32_t* out_sizes,
                                 cudaStream_t stream) {
  if (n_chunks <= 0) return ZMOE_OK;
  ZMOE_CHECK_ARG(n_chunks <= 65535, "lz4_encode: %d chunks in one launch (at most 65535)", n_chunks);
  ZMOE_CHECK_ARG(max_attempts >= 1 && max_attempts <= 65536, "lz4_encode: max_attempts=%d outside [1, 65536]",
                 max_attempts);
  const int hsmem = (int)(kHashSize * sizeof(uint32_t));
  static uint64_t attr_set = 0;                      // devices whose attribute is set
  int dev = 0;
  ZMOE_CUDA_RET(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << (dev & 63)))) {
    ZMOE_CUDA_RET(cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, hsmem));
    attr_set |= 1ull << (dev & 63);
  }
  chain_kernel<<<n_chunks, 32, hsmem, stream>>>(chunks);
  zmoe_status st = launch_status("chain_kernel");
  if (st != ZMOE_OK) return st;
  match_kernel<<<dim3(64, n_chunks), 256, 0, stream>>>(chunks, max_attempts);
  if ((st = launch_status("match_kernel")) != ZMOE_OK) return st;
  emit_kernel<<<n_chunks, 32, 0, stream>>>(chunks, out_sizes);
  return launch_status("emit_kernel");
}

}  // namespace zmoe

// chain links (4), match lengths (4) and offsets (2) per input byte, 16-byte multiple
extern "C" uint64_t zmoe_lz4_encode_scratch_bytes(uint32_t src_size) {
  return ((uint64_t)src_size * 10 + 15) / 16 * 16;
}
