// Offload-side codec: plane split and LZ4 block compression.
//
// Follows the reference's offline conversion:
//  * split_and_extract_from_tensor (runtime/model_offload.py:706-726):
//    exponent plane (u16 >> 7) & 0xFF, sign+mantissa plane
//    ((u16 >> 15) & 1) << 7 | (u16 & 0x7F);
//  * LZ4HCcompressor::compress / LZ4compressor::compress
//    (csrc/tensor_engine/compressors.cpp:105-122, :167-185): LZ4_compress_HC at
//    the configured level, or LZ4_compress_fast at the acceleration level, into
//    an LZ4_compressBound buffer.
// liblz4 is the reference's codec library; it is loaded at run time (the
// image ships the shared library without its header), through its public
// block API only.
#include <dlfcn.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/zmoe.h"

namespace {

typedef int (*bound_fn)(int);
typedef int (*hc_fn)(const char*, char*, int, int, int);
typedef int (*fast_fn)(const char*, char*, int, int, int);

struct Lz4 {
  void* handle = nullptr;
  bound_fn bound = nullptr;
  hc_fn hc = nullptr;
  fast_fn fast = nullptr;
};

Lz4& lz4() {
  static Lz4 l;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"liblz4.so.1", "liblz4.so"};
    for (const char* n : names) {
      l.handle = dlopen(n, RTLD_NOW | RTLD_LOCAL);
      if (l.handle) break;
    }
    if (!l.handle) return;
    l.bound = (bound_fn)dlsym(l.handle, "LZ4_compressBound");
    l.hc = (hc_fn)dlsym(l.handle, "LZ4_compress_HC");
    l.fast = (fast_fn)dlsym(l.handle, "LZ4_compress_fast");
  });
  return l;
}

}  // namespace

extern "C" {

zmoe_status zmoe_split_planes(const uint16_t* bits, uint64_t n, uint8_t* exp, uint8_t* sm) {
  if (n && (!bits || !exp || !sm)) return ZMOE_EINVAL;
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t u = bits[i];
    exp[i] = (uint8_t)((u >> 7) & 0xFF);
    sm[i] = (uint8_t)((((u >> 15) & 1u) << 7) | (u & 0x7Fu));
  }
  return ZMOE_OK;
}

int zmoe_lz4_compress_bound(int n) {
  Lz4& l = lz4();
  return l.bound ? l.bound(n) : -1;
}

int zmoe_lz4_compress(const uint8_t* src, int n, uint8_t* dst, int capacity, int codec, int level) {
  Lz4& l = lz4();
  if (!l.hc || !l.fast || !src || !dst || n < 0) return -1;
  if (codec == ZMOE_CODEC_LZ4HC) return l.hc((const char*)src, (char*)dst, n, capacity, level);
  if (codec == ZMOE_CODEC_LZ4) return l.fast((const char*)src, (char*)dst, n, capacity, level);
  return -1;
}

}  // extern "C"
