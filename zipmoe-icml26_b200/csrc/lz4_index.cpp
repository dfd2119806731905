// Segment index of an LZ4 block (host).
//
// One serial walk over the token stream of a block records, for every
// multiple j*seg_bytes of the output, the first sequence that starts at or
// after it: entry j = (input position of its token, output position).  With
// it, the GPU decoder lets several warps start inside one block at once.  The
// walk follows the LZ4 block format (literal-length and match-length nibbles,
// 255-run extensions, 16-bit offsets, MINMATCH 4, a final literals-only
// sequence); it checks the structure but copies no bytes.
#include <stdint.h>

#include "../../include/zmoe.h"

extern "C" int zmoe_lz4_build_index(const uint8_t* src, uint32_t src_size, uint32_t out_size, uint32_t seg_bytes,
                                    uint32_t* entries, int capacity) {
  if (!src || !entries || seg_bytes == 0 || src_size == 0) return -1;
  const int need = (int)((out_size + seg_bytes - 1) / seg_bytes);
  if (need > capacity) return -2;
  uint64_t ip = 0, op = 0;
  int j = 0;
  while (ip < src_size && op < out_size) {
    while (j < need && (uint64_t)j * seg_bytes <= op) {
      entries[2 * j] = (uint32_t)ip;
      entries[2 * j + 1] = (uint32_t)op;
      ++j;
    }
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
    op += ll;
    if (ip == src_size) break;                 // last sequence
    if (ip + 2 > src_size) return -3;
    const uint32_t off = src[ip] | ((uint32_t)src[ip + 1] << 8);
    ip += 2;
    if (off == 0 || off > op) return -4;
    uint64_t ml = tok & 15;
    if (ml == 15) {
      uint32_t b;
      do {
        if (ip >= src_size) return -3;
        b = src[ip++];
        ml += b;
      } while (b == 255);
    }
    op += ml + 4;
  }
  // Multiples of seg_bytes past the last sequence start: empty segments at the end.
  while (j < need) {
    entries[2 * j] = (uint32_t)ip;
    entries[2 * j + 1] = (uint32_t)(op < out_size ? op : out_size);
    ++j;
  }
  return need;
}
