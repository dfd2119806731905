// extern "C" entry points of libzmoe.so (declared in include/zmoe.h).
#include <stdarg.h>

#include "common.cuh"

namespace zmoe {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

zmoe_status launch_tensor_recover(uint16_t*, const uint8_t*, const uint8_t*, size_t, cudaStream_t);
zmoe_status launch_decode_chunks(const zmoe_chunk*, int, int32_t*, cudaStream_t);
zmoe_status launch_encode_chunks(const zmoe_enc_chunk*, int, int, uint32_t*, cudaStream_t);
zmoe_status launch_router(const zmoe_router_args*, cudaStream_t);
zmoe_status launch_permute(const zmoe_permute_args*, cudaStream_t);
zmoe_status launch_combine(const zmoe_combine_args*, cudaStream_t);
zmoe_status launch_gather_rows(const void*, const int32_t*, int, int, void*, cudaStream_t);

}  // namespace zmoe

extern "C" {

int zmoe_abi_version(void) { return 3; }

const char* zmoe_last_error(void) { return zmoe::g_err; }

zmoe_status zmoe_kernel_error(int32_t* code, int reset) {
  ZMOE_CHECK_ARG(code, "kernel_error: null pointer");
  return zmoe::read_kernel_error(code, reset);
}

zmoe_status zmoe_debug_ffn_wait(long long wait_cycles, int drop_loads) {
  zmoe::set_ffn_wait(wait_cycles, drop_loads);
  return ZMOE_OK;
}

zmoe_status zmoe_tensor_recover(uint16_t* out, const uint8_t* exp, const uint8_t* sm, size_t n,
                                zmoe_stream_t stream) {
  ZMOE_CHECK_ARG(n == 0 || (out && exp && sm), "tensor_recover: null pointer");
  return zmoe::launch_tensor_recover(out, exp, sm, n, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status,
                               zmoe_stream_t stream) {
  ZMOE_CHECK_ARG(n_chunks >= 0, "decode_chunks: negative count");
  ZMOE_CHECK_ARG(n_chunks == 0 || (chunks && status), "decode_chunks: null pointer");
  return zmoe::launch_decode_chunks(chunks, n_chunks, status, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_lz4_encode_chunks(const zmoe_enc_chunk* chunks, int n_chunks, int max_attempts,
                                   uint32_t* out_sizes, zmoe_stream_t stream) {
  ZMOE_CHECK_ARG(n_chunks >= 0, "lz4_encode: negative count");
  ZMOE_CHECK_ARG(n_chunks == 0 || (chunks && out_sizes), "lz4_encode: null pointer");
  return zmoe::launch_encode_chunks(chunks, n_chunks, max_attempts, out_sizes,
                                    reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_router(const zmoe_router_args* a, zmoe_stream_t stream) {
  return zmoe::launch_router(a, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_permute(const zmoe_permute_args* a, zmoe_stream_t stream) {
  return zmoe::launch_permute(a, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_expert_ffn(const zmoe_ffn_args* a, zmoe_stream_t stream) {
  return zmoe::launch_expert_ffn(a, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_gather_rows(const void* src, const int32_t* index, int rows, int row_bytes, void* dst,
                             zmoe_stream_t stream) {
  return zmoe::launch_gather_rows(src, index, rows, row_bytes, dst, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_combine(const zmoe_combine_args* a, zmoe_stream_t stream) {
  return zmoe::launch_combine(a, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
