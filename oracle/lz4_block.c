/*
 * ORACLE — test infrastructure only.  Nothing in the product links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may use it, and only as the checker.
 *
 * Restatement of the LZ4 *block* decoder from the public LZ4 block-format
 * description (token = literal-length nibble | match-length nibble, 255-run
 * length extensions, little-endian 16-bit offset, MINMATCH = 4, the last
 * sequence carries literals only).  The reference decodes each exponent chunk
 * with liblz4's LZ4_decompress_safe_partial(src, dst, csize, osize, osize)
 * (csrc/tensor_engine/compressors.cpp:195-211, call at :201-207); this
 * function has the same contract: decode until `target` output bytes exist,
 * never write past `capacity`, return the number of bytes produced, or a
 * negative value for a malformed block.
 *
 * zmoe_oracle_lz4_encode_chains (below) is the serial statement of the GPU
 * LZ4 block encoder's parse, the bit-exact check of its blocks.
 */
#include <stddef.h>
#include <stdint.h>

int zmoe_oracle_lz4_decode(const uint8_t* src, int src_size, uint8_t* dst,
                           int target, int capacity) {
  const uint8_t* ip = src;
  const uint8_t* const iend = src + src_size;
  uint8_t* op = dst;
  uint8_t* const oend = dst + capacity;
  if (target > capacity) target = capacity;
  if (src_size <= 0) return -1;
  for (;;) {
    if (ip >= iend) return -2;
    unsigned token = *ip++;
    size_t lit = token >> 4;
    if (lit == 15) {
      unsigned b;
      do {
        if (ip >= iend) return -3;
        b = *ip++;
        lit += b;
      } while (b == 255);
    }
    if ((size_t)(iend - ip) < lit) return -4;            /* literal overrun */
    if ((size_t)(oend - op) < lit) {                       /* partial stop */
      size_t room = (size_t)(oend - op);
      for (size_t i = 0; i < room; ++i) op[i] = ip[i];
      op += room;
      return (int)(op - dst);
    }
    for (size_t i = 0; i < lit; ++i) op[i] = ip[i];
    ip += lit;
    op += lit;
    if (op - dst >= target) return (int)(op - dst);
    if (ip == iend) return (int)(op - dst);              /* last sequence */
    if (iend - ip < 2) return -5;
    unsigned off = (unsigned)ip[0] | ((unsigned)ip[1] << 8);
    ip += 2;
    if (off == 0 || (size_t)(op - dst) < off) return -6; /* bad offset */
    size_t mlen = token & 15;
    if (mlen == 15) {
      unsigned b;
      do {
        if (ip >= iend) return -7;
        b = *ip++;
        mlen += b;
      } while (b == 255);
    }
    mlen += 4;
    const uint8_t* match = op - off;
    size_t room = (size_t)(oend - op);
    size_t n = mlen < room ? mlen : room;
    for (size_t i = 0; i < n; ++i) op[i] = match[i];     /* overlap-safe */
    op += n;
    if (op - dst >= target) return (int)(op - dst);
    if (n < mlen) return (int)(op - dst);
  }
}

/* Recombine the exponent plane and the sign+mantissa plane into BF16 bit
 * patterns: out = (sm>>7)<<15 | exp<<7 | (sm & 0x7F)
 * (csrc/kernels/tensor_recover.cu:25-30). */
void zmoe_oracle_recombine(const uint8_t* exp, const uint8_t* sm, uint16_t* out,
                           size_t n) {
  for (size_t i = 0; i < n; ++i) {
    unsigned s = sm[i];
    out[i] = (uint16_t)(((s >> 7) << 15) | ((unsigned)exp[i] << 7) | (s & 0x7F));
  }
}

/* Serial statement of the GPU LZ4 block encoder's parse (the reference
 * compresses with liblz4's LZ4_compress_HC, csrc/tensor_engine/compressors.cpp:105-122;
 * the GPU encoder is a different LZ4 encoder whose blocks any LZ4 decoder
 * reads).  Positions are visited in order, so the hash chains are those of a
 * serial insertion:
 *   prev[i]  latest j < i with hash(4 bytes at j) == hash(4 bytes at i),
 *            hash = (le32 * 2654435761) >> 17;
 *   match[i] the longest of at most `attempts` chain candidates inside the
 *            64 KiB window (searched up to 1024 bytes; the nearest wins ties),
 *            none reaching into the last 5 bytes, none starting in the last 12,
 *            none crossing a 16 KiB segment boundary (the GPU parses the
 *            segments in parallel);
 *   parse    greedy with one step of lazy evaluation (a match is put off by
 *            one byte when the next position, if it may start a match, has a
 *            longer one); a match searched to 1024 bytes is extended while the
 *            bytes repeat.
 * Returns the block size, or 0 when it would not fit `capacity`, or -1 when
 * scratch cannot be allocated. */
#include <stdlib.h>
#include <string.h>

#define ENC_NONE 0xFFFFFFFFu
#define ENC_LEN_CAP 1024u
#define ENC_SEGMENT 16384u

static uint32_t enc_rd4(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

typedef struct { uint8_t* dst; uint32_t op, cap; int ok; } enc_out;

static void enc_byte(enc_out* o, uint32_t v) {
  if (o->op < o->cap) o->dst[o->op] = (uint8_t)v; else o->ok = 0;
  o->op++;
}

static void enc_run(enc_out* o, uint32_t rest) {
  while (rest >= 255) { enc_byte(o, 255); rest -= 255; }
  enc_byte(o, rest);
}

static void enc_sequence(enc_out* o, const uint8_t* lit, uint32_t ll, uint32_t off, uint32_t ml) {
  uint32_t mcode = ml ? ml - 4 : 0;
  enc_byte(o, ((ll >= 15 ? 15u : ll) << 4) | (ml ? (mcode >= 15 ? 15u : mcode) : 0u));
  if (ll >= 15) enc_run(o, ll - 15);
  for (uint32_t k = 0; k < ll; ++k) enc_byte(o, lit[k]);
  if (!ml) return;
  enc_byte(o, off & 0xFF);
  enc_byte(o, off >> 8);
  if (mcode >= 15) enc_run(o, mcode - 15);
}

int zmoe_oracle_lz4_encode_chains(const uint8_t* src, uint32_t n, uint8_t* dst, uint32_t capacity,
                                  int attempts) {
  uint32_t* head = (uint32_t*)malloc(sizeof(uint32_t) << 15);
  uint32_t* prev = (uint32_t*)malloc(sizeof(uint32_t) * ((size_t)n + 1));
  uint32_t* mlen = (uint32_t*)malloc(sizeof(uint32_t) * ((size_t)n + 1));
  uint16_t* moff = (uint16_t*)malloc(sizeof(uint16_t) * ((size_t)n + 1));
  int ret = -1;
  if (!head || !prev || !mlen || !moff) goto done;
  for (uint32_t h = 0; h < (1u << 15); ++h) head[h] = ENC_NONE;
  for (uint32_t i = 0; i < n; ++i) {
    prev[i] = ENC_NONE;
    if (i + 4 <= n) {
      uint32_t h = (enc_rd4(src + i) * 2654435761u) >> 17;
      prev[i] = head[h];
      head[h] = i;
    }
  }
  for (uint32_t i = 0; i < n; ++i) {
    uint32_t best = 0, best_off = 0;
    uint32_t seg_end = (i / ENC_SEGMENT + 1) * ENC_SEGMENT;
    if (seg_end > n) seg_end = n;
    if (i + 12 <= n && seg_end - i >= 4) {
      uint32_t max_len = n - 5 - i;
      if (max_len > ENC_LEN_CAP) max_len = ENC_LEN_CAP;
      if (max_len > seg_end - i) max_len = seg_end - i;
      uint32_t key = enc_rd4(src + i), cand = prev[i];
      for (int a = 0; a < attempts && cand != ENC_NONE; ++a) {
        if (cand >= i || i - cand > 65535) break;
        if (enc_rd4(src + cand) == key) {
          uint32_t len = 4;
          while (len < max_len && src[cand + len] == src[i + len]) ++len;
          if (len > best) {
            best = len;
            best_off = i - cand;
            if (len >= max_len) break;
          }
        }
        cand = prev[cand];
      }
    }
    mlen[i] = best >= 4 ? best : 0;
    moff[i] = (uint16_t)best_off;
  }
  {
    enc_out o = {dst, 0, capacity, 1};
    uint32_t i = 0, anchor = 0;
    while (i + 12 <= n && o.ok) {
      uint32_t len = mlen[i];
      if (len < 4 || (i + 13 <= n && mlen[i + 1] > len)) { ++i; continue; }
      uint32_t off = moff[i], ml = len;
      if (ml == ENC_LEN_CAP) {
        uint32_t end = (i / ENC_SEGMENT + 1) * ENC_SEGMENT;
        if (end > n - 5) end = n - 5;
        while (i + ml < end && src[i + ml] == src[i + ml - off]) ++ml;
      }
      enc_sequence(&o, src + anchor, i - anchor, off, ml);
      i += ml;
      anchor = i;
    }
    if (o.ok) enc_sequence(&o, src + anchor, n - anchor, 0, 0);
    ret = o.ok ? (int)o.op : 0;
  }
done:
  free(head); free(prev); free(mlen); free(moff);
  return ret;
}
