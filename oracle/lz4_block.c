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
