// Slice index of an LZ4 block (host).
//
// One serial walk over the token stream of a block records, for every
// multiple j*slice_bytes of the output, the sequence that CONTAINS output byte
// j*slice_bytes: entry j = (input position of its token, output position where
// it starts).  With it the GPU decoder gives every lane its own slice of
// slice_bytes output bytes to parse: the lane starts at that token, skips to
// byte j*slice_bytes and stops at the next slice.  The walk follows the LZ4
// block format (literal-length and match-length nibbles, 255-run extensions,
// 16-bit offsets, MINMATCH 4, a final literals-only sequence); it checks the
// structure but copies no bytes.
#include <stdint.h>

#include "../../include/zmoe.h"

extern "C" int zmoe_lz4_build_index(const uint8_t* src, uint32_t src_size, uint32_t out_size, uint32_t seg_bytes,
                                    uint32_t* entries, int capacity) {
  if (!src || !entries || seg_bytes == 0 || src_size == 0) return -1;
  const int need = (int)((out_size + seg_bytes - 1) / seg_bytes);
  if (need > capacity) return -2;
  uint64_t ip = 0, op = 0;
  int j = 0;
  while (ip < src_size && j < need) {
    const uint64_t tok_pos = ip;
    const uint32_t tok = src[ip++];
    uint64_t ll = tok >> 4;
    if (ll == 15) {
      uint32_t b;
      do {
        if (ip >= src_size) return -3;
        b = src[ip++];
        ll += b;
      } while (b == 255);
    }
    if (ip + ll > src_size) return -3;
    ip += ll;
    uint64_t ml = 0;
    if (ip < src_size) {
      if (ip + 2 > src_size) return -3;
      const uint32_t off = src[ip] | ((uint32_t)src[ip + 1] << 8);
      ip += 2;
      if (off == 0 || off > op + ll) return -4;
      ml = tok & 15;
      if (ml == 15) {
        uint32_t b;
        do {
          if (ip >= src_size) return -3;
          b = src[ip++];
          ml += b;
        } while (b == 255);
      }
      ml += 4;
    }
    const uint64_t end = op + ll + ml;
    // every slice boundary inside [op, end) belongs to this sequence
    while (j < need && (uint64_t)j * seg_bytes < end) {
      entries[2 * j] = (uint32_t)tok_pos;
      entries[2 * j + 1] = (uint32_t)op;
      ++j;
    }
    op = end;
  }
  if (j < need) return -5;   // the block ends before out_size bytes
  return need;
}
