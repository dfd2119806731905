/*
 * zmoe.h — C ABI of the B200 (sm_100a) expert hot path of ZipMoE.
 *
 * Every entry point takes plain pointers and sizes, works on caller-owned
 * device memory, is asynchronous on the given stream, and returns a
 * zmoe_status.  Per-item device status words report data errors (a malformed
 * LZ4 block, an output overflow) without trapping the GPU.
 *
 * Each declaration names the reference interface it replaces (paths are
 * relative to the reference project root).
 */
#ifndef ZMOE_H_
#define ZMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Binary-compatible with cudaStream_t. */
typedef struct CUstream_st* zmoe_stream_t;

typedef enum zmoe_status {
  ZMOE_OK = 0,
  ZMOE_EINVAL = 1,      /* bad argument (null pointer, unsupported size) */
  ZMOE_ECUDA = 2,       /* a CUDA runtime call failed */
  ZMOE_EUNSUPPORTED = 3,/* shape outside what the kernels implement */
  ZMOE_ENOMEM = 4,
  ZMOE_ENCCL = 5,
  ZMOE_EKERNEL = 6      /* a kernel gave up a bounded wait: that call's outputs are incomplete */
} zmoe_status;

/* Per-chunk decode status written by zmoe_decode_chunks. */
enum {
  ZMOE_CHUNK_OK = 0,
  ZMOE_CHUNK_BAD_OFFSET = 1,     /* zero offset or offset before the chunk start */
  ZMOE_CHUNK_INPUT_OVERRUN = 2,  /* a length runs past the end of the block */
  ZMOE_CHUNK_SHORT_OUTPUT = 3,   /* the block ended before out_size bytes */
  ZMOE_CHUNK_BAD_DESC = 4        /* null pointer or zero-sized block */
};

/* Version of this ABI. */
int zmoe_abi_version(void);

/* Average SM clock over a window, measured on the GPU by one thread: out is a
 * device array of 2 uint64, receiving the SM cycles counted and the
 * nanoseconds elapsed (MHz = out[0] * 1000 / out[1]).  Runs on `stream` next
 * to other work, so a benchmark can record the clock under load without a
 * driver query.  No counterpart in the reference. */
zmoe_status zmoe_clock_probe(uint64_t* out, uint64_t window_ns, zmoe_stream_t stream);

/* Human-readable text of the last error recorded on the calling thread. */
const char* zmoe_last_error(void);

/* Device-wide error word of the tcgen05 expert-FFN kernels on the current
 * device: 0, or 1 once a launch gave up one of its bounded mbarrier waits
 * (it then drained its own copies, freed its TMEM and returned, leaving its
 * outputs incomplete).  Synchronous; reset != 0 clears the word after reading.
 * No counterpart in the reference, whose libtorch FFN has no device waits. */
zmoe_status zmoe_kernel_error(int32_t* code, int reset);
/* Test hook for the error path above (no counterpart in the reference): later
 * expert-FFN launches from this process use wait_cycles (clock64 cycles; <= 0
 * restores the default of about 2 s) as their wait limit, and with
 * drop_loads != 0 their TMA producer issues no loads, so that the first MMA
 * wait runs out and the launch returns through the error path.  Nothing
 * faults or hangs: every wait stays bounded. */
zmoe_status zmoe_debug_ffn_wait(long long wait_cycles, int drop_loads);

/* --------------------------------------------------------------------------
 * Plane recombine.
 * Replaces zipmoe_launch_tensor_recover (csrc/kernels/tensor_recover.hpp:14-20,
 * kernel csrc/kernels/tensor_recover.cu:12-43):
 *   out[i] = (sm[i] >> 7) << 15 | exp[i] << 7 | (sm[i] & 0x7F)
 * n is a 64-bit count (the reference kernel takes a 32-bit int).
 * ------------------------------------------------------------------------ */
zmoe_status zmoe_tensor_recover(uint16_t* out, const uint8_t* exp, const uint8_t* sm,
                                size_t n, zmoe_stream_t stream);

/* --------------------------------------------------------------------------
 * Fused LZ4-block decode + recombine.
 * Replaces, per exponent chunk, LZ4_decompress_safe_partial(src, dst, csize,
 * osize, osize) in LZ4compressor/LZ4HCcompressor::decompress
 * (csrc/tensor_engine/compressors.cpp:133-149,195-211) as driven by
 * TensorEngine::io_decompress_mov_submit (csrc/tensor_engine/tensor_engine.cpp:421-474),
 * followed by the recombine launch of SetModuleMemoryFromDiskGrouped
 * (csrc/topology/model_topology.cpp:574-580).  The decoded exponent bytes never
 * leave the SM: each one is merged with its sign+mantissa byte and written as
 * BF16 straight into the destination slot.
 * ------------------------------------------------------------------------ */
#define ZMOE_SLICE_BYTES 256      /* output bytes per slice-index entry */
#define ZMOE_MAP_ENTRIES 65536    /* map entries per 64 KiB region of output */

typedef struct zmoe_chunk {
  const uint8_t* src;   /* LZ4 block, device memory */
  const uint8_t* sm;    /* sign+mantissa bytes of this chunk's elements */
  uint16_t* dst;        /* BF16 output of this chunk's elements */
  const uint32_t* index;/* device [n_index][2] slice index from zmoe_lz4_build_index, or NULL */
  uint32_t* map;        /* device scratch of zmoe_decode_scratch_bytes(out_size), 16-byte aligned (with index) */
  uint32_t src_size;    /* compressed bytes */
  uint32_t out_size;    /* exponent bytes = elements (original_sizes[c]) */
  uint32_t n_index;     /* entries in index */
  uint32_t seg_bytes;   /* output bytes per index entry: ZMOE_SLICE_BYTES */
} zmoe_chunk;

/* chunks and status are device arrays of n_chunks entries.  Indexed chunks
 * are decoded by two launches on the stream: the map kernel (one thread per
 * 256-byte slice, 16 CTAs per chunk) writes the source of every output byte
 * into zmoe_chunk.map; the resolve kernel (one CTA per chunk) follows the
 * sources in 2 KiB steps through a 64 KiB shared-memory ring and writes the
 * recombined BF16.  A chunk without an index is decoded serially by one warp.
 * status[c] is always written (ZMOE_CHUNK_OK or the first error found). */
zmoe_status zmoe_decode_chunks(const zmoe_chunk* chunks, int n_chunks, int32_t* status,
                               zmoe_stream_t stream);
/* Scratch bytes an indexed chunk of out_size exponent bytes needs in
 * zmoe_chunk.map: one source-map entry per output byte (whole 64 KiB regions)
 * and one status word per region. */
uint64_t zmoe_decode_scratch_bytes(uint32_t out_size);

/* Host: slice index of one LZ4 block (no counterpart in the reference; the
 * reference decodes each block serially on one CPU thread).  Entry j =
 * (input position of the token, output position where it starts) of the
 * sequence that contains output byte j * seg_bytes; ceil(out_size / seg_bytes)
 * entries are written to entries[2 * j .. 2 * j + 1].  Returns the entry
 * count, or a negative value for a malformed block (-3 overrun, -4 bad offset,
 * -5 fewer than out_size bytes) or too small a capacity (-2). */
int zmoe_lz4_build_index(const uint8_t* src, uint32_t src_size, uint32_t out_size, uint32_t seg_bytes,
                         uint32_t* entries, int capacity);

/* --------------------------------------------------------------------------
 * Router: logits, softmax and top-k of one MoE layer.
 * Replaces Qwen2MoEBlock.__prepare_expert_route (customized/qwen.py:44-54),
 * MoEGate.forward greedy branch (models/deepseek/modeling_deepseek.py:424-476)
 * and the transformers<4.47 SwitchTransformersTop1Router used by
 * customized/switch_transformers.py:72-73.
 * Logits accumulate in fp32 in a fixed order (lane l of 32 sums h = 256j+8l+i,
 * xor-butterfly fold); ties in top-k go to the lower expert index.
 * ------------------------------------------------------------------------ */
enum { ZMOE_ROUTE_QWEN = 0, ZMOE_ROUTE_DEEPSEEK = 1, ZMOE_ROUTE_SWITCH = 2 };

typedef struct zmoe_router_args {
  const uint16_t* x;          /* [T, H] BF16 */
  const uint16_t* w;          /* [E, H] BF16 router weight */
  const float* bias;          /* [E] fp32 logit bias or NULL */
  const uint16_t* w_shared_gate; /* [H] BF16 (Qwen shared-expert gate) or NULL */
  int T, H, E, k;
  int mode;                   /* ZMOE_ROUTE_* */
  int norm_topk_prob;         /* Qwen/DeepSeek renormalisation flag */
  float scaling;              /* DeepSeek routed_scaling_factor */
  float* logits;              /* [T, E] fp32 out (may be NULL) */
  int32_t* topk_idx;          /* [T, k] out */
  float* topk_w;              /* [T, k] out combine weights */
  float* shared_gate;         /* [T] out sigmoid gate, when w_shared_gate != NULL */
} zmoe_router_args;

zmoe_status zmoe_router(const zmoe_router_args* a, zmoe_stream_t stream);

/* --------------------------------------------------------------------------
 * Permute: group the routed (token, slot) pairs by expert, tokens ascending
 * inside an expert, and gather the activation rows.
 * Replaces the boolean-mask gather hidden_states_.index({token_indices}) of
 * ExpertDispatcher::GPUFetchFunc (csrc/dispatcher/expert_dispatcher.cpp:326-330)
 * and the per-expert counts of ExpertExecutor.dispatch_local
 * (experts/expert_executor.py:45-49).  For Switch (capacity > 0) a token is
 * dropped when its expert already has `capacity` earlier tokens in the same
 * sequence of length seq_len (the cumsum mask of the Top1 router).
 * ------------------------------------------------------------------------ */
typedef struct zmoe_permute_args {
  int32_t* topk_idx;          /* [T, k] in; dropped entries are set to -1 */
  const uint16_t* x;          /* [T, H] BF16 */
  int T, H, E, k;
  int capacity, seq_len;      /* capacity 0 = unlimited */
  int32_t* counts;            /* [E] out tokens per expert */
  int32_t* offsets;           /* [E + 1] out exclusive prefix */
  int32_t* row_of;            /* [T, k] out permuted row or -1 */
  int32_t* token_of_row;      /* [T * k] out */
  uint16_t* xp;               /* [T * k, H] out gathered rows */
} zmoe_permute_args;

zmoe_status zmoe_permute(const zmoe_permute_args* a, zmoe_stream_t stream);

/* --------------------------------------------------------------------------
 * Grouped expert FFN over the permuted rows.
 * Replaces DeepSeekMoEDenseActDense::forward (csrc/dispatcher/expert_module.cpp:39-50)
 * and SwitchTransformersDenseActDense::forward (:67-78) run one expert at a
 * time by ExpertDispatcher::GPUExecFunc (expert_dispatcher.cpp:354-427).
 * kind 0: y = bf16(bf16(silu(x Wg^T) * (x Wu^T)) Wd^T) ; kind 1: y = bf16(bf16(relu(x Wi^T)) Wo^T):
 * fp32 accumulation, the intermediate and the output each rounded to BF16
 * once (the reference's libtorch FFN returns BF16 rows).
 * w[g*3 + {0,1,2}] are the device pointers of group g's matrices (row-major
 * [I, H], [I, H], [H, I]; for kind 1 w[g*3+0] = wi [I, H], w[g*3+2] = wo [H, I]).
 * Rows of group g are offsets[g] .. offsets[g+1] of x; NULL offsets means one
 * group of rows_total rows.  y is BF16 [rows, H]; h is BF16 scratch [rows, I].
 * ------------------------------------------------------------------------ */
typedef struct zmoe_ffn_args {
  const uint16_t* x;          /* [rows, H] BF16 */
  const uint16_t* const* w;   /* HOST array [G * 3] of device weight pointers (the launch builds one
                                 TMA descriptor per matrix on the host); a group's pointers are all
                                 set (w[1] may be NULL for kind 1) or all NULL (group skipped) */
  const int32_t* offsets;     /* [G + 1] device or NULL */
  int G, rows_total, H, I, kind;
  uint16_t* h;                /* [rows, I] BF16 scratch */
  uint16_t* y;                /* [rows, H] BF16 out */
} zmoe_ffn_args;

zmoe_status zmoe_expert_ffn(const zmoe_ffn_args* a, zmoe_stream_t stream);

/* Same computation for callers that cannot allocate device memory (no
 * counterpart in the reference).  Runtimes that own all device memory through
 * their own pool, or that must not call cudaMalloc/cudaFree mid-step (a
 * cudaFree synchronises the device), cannot provide the h scratch buffer;
 * here a->h is ignored and the intermediate lives in a file-scope device array
 * of 16 Mi BF16 elements (32 MiB, held on every GPU that loads the library
 * until exit).  rows_total * I above that is rejected (ZMOE_EUNSUPPORTED).
 * Calls no cudaMalloc, cudaFree or allocating routine.  All calls share the
 * array, which keeps the last call's contents; calls that overlap on the GPU
 * race and must be serialised.  The first call on a device looks up the
 * array's address with that device current; make it before any stream capture. */
zmoe_status zmoe_expert_ffn_noalloc(const zmoe_ffn_args* a, zmoe_stream_t stream);

/* --------------------------------------------------------------------------
 * Combine: gate-weighted sum of the expert rows plus the shared expert.
 * Replaces the Python combine loops customized/qwen.py:89-100,
 * customized/deepseek.py:103-115 and customized/switch_transformers.py:83-87.
 * mode QWEN/DEEPSEEK: out[t] = sum_j w[t,j] y[row_of[t,j]] + g[t] * ysh[t]
 *   (g = shared_gate[t], or 1 when shared_gate is NULL; no ysh term when NULL).
 * mode SWITCH: out[t] = w[t,0] * (row_of[t,0] >= 0 ? y[row_of[t,0]] : x[t]).
 * fp32 accumulation, one BF16 rounding.
 * ------------------------------------------------------------------------ */
typedef struct zmoe_combine_args {
  const uint16_t* y;          /* [rows, H] BF16 expert rows */
  const uint16_t* y_shared;   /* [T, H] BF16 shared-expert rows, or NULL */
  const float* shared_gate;   /* [T] or NULL */
  const int32_t* row_of;      /* [T, k] */
  const float* topk_w;        /* [T, k] */
  const uint16_t* x;          /* [T, H] (Switch pass-through) */
  int T, H, k, mode;
  uint16_t* out;              /* [T, H] BF16 */
} zmoe_combine_args;

zmoe_status zmoe_combine(const zmoe_combine_args* a, zmoe_stream_t stream);

/* Row gather dst[r] = src[index[r]], r < rows, for rows of row_bytes bytes (a
 * multiple of 16; src and dst 16-byte aligned).  Regroups token rows received
 * from other ranks by expert, and back, under expert parallelism; the
 * reference gathers an expert's rows with a libtorch boolean index
 * (csrc/dispatcher/expert_dispatcher.cpp:326-330). */
zmoe_status zmoe_gather_rows(const void* src, const int32_t* index, int rows, int row_bytes, void* dst,
                             zmoe_stream_t stream);

/* --------------------------------------------------------------------------
 * Offload-side codec (host).
 * zmoe_split_planes replaces split_and_extract_from_tensor
 * (runtime/model_offload.py:706-726); zmoe_lz4_compress replaces
 * LZ4HCcompressor::compress / LZ4compressor::compress
 * (csrc/tensor_engine/compressors.cpp:105-122, :167-185) and returns the block
 * size, or a value <= 0 on failure.
 * ------------------------------------------------------------------------ */
enum { ZMOE_CODEC_LZ4 = 0, ZMOE_CODEC_LZ4HC = 1 };

zmoe_status zmoe_split_planes(const uint16_t* bits, uint64_t n, uint8_t* exp, uint8_t* sm);
int zmoe_lz4_compress_bound(int n);
int zmoe_lz4_compress(const uint8_t* src, int n, uint8_t* dst, int capacity, int codec, int level);

/* --------------------------------------------------------------------------
 * Offload-side codec on the GPU.
 * zmoe_lz4_encode_chunks replaces the LZ4HCcompressor::compress calls
 * (csrc/tensor_engine/compressors.cpp:105-122) that TensorEngine::PipelineCompress
 * runs on one CPU thread per exponent chunk: every chunk of a launch is encoded
 * at once.  The blocks are valid LZ4 blocks (any LZ4 decoder restores the
 * chunk); they are not byte-identical to liblz4's.
 * ------------------------------------------------------------------------ */
typedef struct zmoe_enc_chunk {
  const uint8_t* src;    /* device: the chunk's exponent bytes */
  uint8_t* dst;          /* device: the LZ4 block */
  void* scratch;         /* device, 16-byte aligned: zmoe_lz4_encode_scratch_bytes(src_size) bytes */
  uint32_t src_size;     /* bytes in src */
  uint32_t dst_capacity; /* bytes available at dst (zmoe_lz4_compress_bound(src_size) always suffices) */
} zmoe_enc_chunk;

/* chunks (n_chunks entries) and out_sizes are device arrays.  max_attempts
 * (1..65536) bounds the hash-chain candidates tried per position, as LZ4HC's
 * compression level does.  out_sizes[c] = block size, or 0 when the block did
 * not fit dst_capacity or a pointer of chunk c was null or misaligned. */
zmoe_status zmoe_lz4_encode_chunks(const zmoe_enc_chunk* chunks, int n_chunks, int max_attempts,
                                   uint32_t* out_sizes, zmoe_stream_t stream);
/* Scratch bytes a chunk of src_size bytes needs: chain link, match length
 * and match offset per input byte, and a 32-byte record per 16 KiB. */
uint64_t zmoe_lz4_encode_scratch_bytes(uint32_t src_size);

/* --------------------------------------------------------------------------
 * MoE-layer engine (opaque handle).
 * Re-targets, for one layer, the reference's runtime around the hot path:
 * ZipMoEPrefetchHandle's stores and pools (csrc/prefetch/zipmoe_prefetch_handle.cpp:33-108),
 * ZipMoECacheHandle::ProactiveDecision and its slot policies
 * (csrc/memory/cache.cpp:226-270, :445-690), TensorEngine::ToWorkers /
 * ZipMoESchedulerFunc (csrc/tensor_engine/tensor_engine.cpp:515-669) and the
 * ExpertDispatcher fetch/exec/output loop (csrc/dispatcher/expert_dispatcher.cpp:285-515).
 * Compressed experts stay resident in HBM in the reference's storage form
 * (LZ4 exponent chunks + raw sign+mantissa plane); cache_slots decoded experts
 * stay resident; misses are decoded by zmoe_decode_chunks into cache slots
 * (NORMAL) or transient slots (EVICT) before the grouped FFN runs.
 * ------------------------------------------------------------------------ */
typedef struct zmoe_layer zmoe_layer;

enum { ZMOE_CACHE_ZIPMOE = 0, ZMOE_CACHE_LFU = 1, ZMOE_CACHE_LRU = 2, ZMOE_CACHE_FIFO = 3 };

typedef struct zmoe_layer_config {
  int hidden, num_experts, inter, topk;
  int kind;                   /* 0 SwiGLU (Qwen/DeepSeek), 1 ReLU (Switch) */
  int route_mode;             /* ZMOE_ROUTE_* */
  int norm_topk_prob;
  float scaling;              /* DeepSeek routed_scaling_factor */
  int shared_inter;           /* shared-expert intermediate size, 0 = none */
  int capacity, seq_len;      /* Switch capacity per sequence of seq_len tokens */
  int max_tokens;             /* workspace is sized for this many tokens */
  int cache_slots;            /* decoded experts kept resident */
  int transient_slots;        /* decode slots for misses; 0 = num_experts - cache_slots */
  int cache_policy;           /* ZMOE_CACHE_* victim selection */
  double state_margin;        /* hyperparam_state_margin of the NORMAL threshold */
  int sm_slots;               /* host store: experts whose sign+mantissa planes stay in HBM (the SMCACHE
                                 pool of ZipMoECacheHandle, csrc/memory/cache.cpp:122-123, 369-401) */
} zmoe_layer_config;

typedef struct zmoe_layer_stats {
  uint64_t forwards, tokens, hits, misses, evictions;
  uint64_t decoded_experts, decoded_chunks, decoded_bytes, decode_launches;
  uint64_t launches, decode_errors, store_bytes;
  /* filled when timing is on: CUDA-event durations on the launch stream */
  uint64_t decode_ns, decode_timed_bytes, decode_timed_launches, ffn_ns, ffn_timed_launches;
  uint64_t host_copy_bytes;   /* host tier: compressed bytes copied to the GPU for decodes */
  uint64_t sm_resident_tensors; /* host tier: tensors decoded with their sign+mantissa plane resident in HBM */
} zmoe_layer_stats;

zmoe_status zmoe_layer_create(const zmoe_layer_config* cfg, zmoe_layer** out);
zmoe_status zmoe_layer_destroy(zmoe_layer* layer);
/* Host pointers; copied to HBM.  bias ([E] fp32) and w_shared_gate ([H] BF16) may be NULL. */
zmoe_status zmoe_layer_set_router(zmoe_layer* layer, const uint16_t* w_router, const float* bias,
                                  const uint16_t* w_shared_gate);
zmoe_status zmoe_layer_set_shared(zmoe_layer* layer, const uint16_t* gate, const uint16_t* up,
                                  const uint16_t* down);
/* One expert tensor in the reference's storage form, from host memory: the LZ4
 * blocks of its exponent chunks and its raw sign+mantissa plane (what
 * TensorEngine::PipelineCompress writes, tensor_engine.cpp:168-220). */
zmoe_status zmoe_layer_load_expert(zmoe_layer* layer, int expert, int tensor, const uint8_t* const* blocks,
                                   const uint32_t* block_sizes, const uint32_t* original_sizes, int n_chunks,
                                   const uint8_t* sm, uint64_t numel);
/* Where the compressed experts live, chosen before the first
 * zmoe_layer_load_expert: ZMOE_STORE_DEVICE (default, HBM) or ZMOE_STORE_HOST
 * (pinned host memory; every decode first copies each missed tensor's
 * compressed blocks, index and sign+mantissa plane into a device staging area
 * on the stream).  The host tier is for models whose compressed experts do not
 * fit the GPU; a miss then costs a PCIe copy of the compressed tensor.  It
 * replaces the reference's per-miss reads of the stored planes
 * (tensor_engine.cpp:380-417, pread into pinned docks).  With sm_slots > 0 the
 * host tier keeps a pool of sign+mantissa planes in HBM (the reference's
 * SMCACHE state): a miss ranked, by the layer's token counts, below
 * cache_slots + sm_slots + margin * E but not admitted to a decoded slot gets
 * (or keeps) its planes in the pool, and its later misses copy only the
 * exponent blocks and index (about a third of the bytes). */
enum { ZMOE_STORE_DEVICE = 0, ZMOE_STORE_HOST = 1 };
zmoe_status zmoe_layer_set_store(zmoe_layer* layer, int where);
/* Decode the given experts into free cache slots now. */
zmoe_status zmoe_layer_warm_cache(zmoe_layer* layer, const int* experts, int n, zmoe_stream_t stream);
/* x, out: device [T, H] BF16.  Synchronises once on the stream to read the
 * per-expert token counts. */
zmoe_status zmoe_layer_forward(zmoe_layer* layer, const uint16_t* x, int T, uint16_t* out, zmoe_stream_t stream);
/* Expert stage alone, for expert parallelism (the caller routes, permutes and
 * exchanges rows): x_rows device [rows, H] BF16 grouped by this layer's
 * experts, counts_host[e] rows of expert e (host array, summing to rows <=
 * max_tokens * topk); applies the cache decision, decodes misses and runs the
 * grouped FFN into y, device [rows, H] BF16.  Router and shared-expert weights
 * are not used.  Replaces, for the experts one rank owns,
 * ExpertDispatcher::EnqueueExpert .. Wait (csrc/dispatcher/expert_dispatcher.cpp:149-217,285-515).
 * Does not wait for the stream: it waits only for this layer's own earlier
 * copies and decodes (events). */
zmoe_status zmoe_layer_experts(zmoe_layer* layer, const uint16_t* x_rows, const int32_t* counts_host, int rows,
                               uint16_t* y, zmoe_stream_t stream);
/* Same with host buffers (pinned for full speed); returns after out_host is written. */
zmoe_status zmoe_layer_forward_host(zmoe_layer* layer, const uint16_t* x_host, int T, uint16_t* out_host,
                                    zmoe_stream_t stream);
/* Pipelined form of zmoe_layer_forward_host (no counterpart in the
 * reference, whose layer runs synchronously per call): queues the input copy, the
 * forward on `stream` and the output copy, and returns once the forward is
 * launched (it waits only for this step's expert counts, like
 * zmoe_layer_forward).  Copies run on the layer's own copy streams through two
 * device staging slots, so one step's copies overlap the neighbouring steps'
 * compute.  x_host must stay unchanged and out_host unread until
 * zmoe_layer_join_host and a wait on its stream. */
zmoe_status zmoe_layer_submit_host(zmoe_layer* layer, const uint16_t* x_host, int T, uint16_t* out_host,
                                   zmoe_stream_t stream);
/* Makes `stream` wait (without blocking the host) until the output copies of
 * every submitted step have completed. */
zmoe_status zmoe_layer_join_host(zmoe_layer* layer, zmoe_stream_t stream);
/* Wait for the stream and report any decode error of earlier forwards
 * (ZMOE_EINVAL) or an expert-FFN launch that gave up a wait (ZMOE_EKERNEL).
 * zmoe_layer_forward and zmoe_layer_experts report both too, for earlier
 * calls whose work has finished by then. */
zmoe_status zmoe_layer_sync(zmoe_layer* layer, zmoe_stream_t stream);
zmoe_status zmoe_layer_get_stats(const zmoe_layer* layer, zmoe_layer_stats* out);
zmoe_status zmoe_layer_reset_stats(zmoe_layer* layer);
/* Record CUDA events around every decode and routed-FFN launch (stats *_ns). */
zmoe_status zmoe_layer_set_timing(zmoe_layer* layer, int enable);
zmoe_status zmoe_layer_cached_experts(const zmoe_layer* layer, int32_t* experts, int cap, int* n);
/* Decode experts into cache slots ahead of use (victims by the cache policy,
 * never one of `experts`); returns without waiting for the decode.  Replaces
 * ExpertDispatcher::SubmitPrefetch / EnqueuePrefetch
 * (csrc/dispatcher/expert_dispatcher.cpp:220-277). */
zmoe_status zmoe_layer_prefetch(zmoe_layer* layer, const int* experts, int n, zmoe_stream_t stream);
/* Per-expert token counts of the layer's last forward or expert stage
 * (counts[e], e < cap; n receives the number of experts).  The input of a
 * next-layer predictor: the reference's ExpertExecutor records each layer's
 * activated experts for ExpertPredictor (experts/expert_executor.py:68-83). */
zmoe_status zmoe_layer_last_counts(const zmoe_layer* layer, int32_t* counts, int cap, int* n);
/* Zero the per-expert token counts behind the cache decision (the admission
 * rank and the LFU/ZipMoE victim keys); replaces
 * ZipMoECacheHandle::reset_global_access_counts (csrc/memory/cache.cpp). */
zmoe_status zmoe_layer_reset_access_counts(zmoe_layer* layer);

/* --------------------------------------------------------------------------
 * Expert-parallel layer over NCCL (one process per GPU).
 * Rank r owns experts [r*E/P, (r+1)*E/P) in its own zmoe_layer (created with
 * those E_r experts and max_tokens >= P * the per-rank max_tokens below);
 * router, shared expert and tokens are data-parallel.  A forward routes and
 * permutes the rank's tokens, sends per-expert counts and then the BF16 rows
 * to the experts' ranks (grouped ncclSend/ncclRecv), runs the local experts
 * (zmoe_layer_experts: cache decision, miss decode, grouped FFN), returns the
 * BF16 rows and combines them with the shared expert, which runs on a side
 * stream during the exchange.  The host waits once per forward, for the
 * counts.  Replaces, for the ranks of an expert-parallel deployment, the
 * reference's per-rank ExpertExecutor.dispatch_local (experts/expert_executor.py:40-84)
 * and the exchange around it.  nccl_comm is an ncclComm_t of the world ranks
 * created by the NCCL library already loaded in the process (for example
 * torch's ProcessGroupNCCL._comm_ptr()); every rank calls zmoe_ep_forward in
 * the same order.  A world of 1 needs no communicator.
 * ------------------------------------------------------------------------ */
typedef struct zmoe_ep zmoe_ep;

typedef struct zmoe_ep_config {
  zmoe_layer_config layer;    /* the whole layer: all E experts; max_tokens per rank; cache fields unused */
  int rank, world;
  void* nccl_comm;            /* ncclComm_t */
} zmoe_ep_config;

zmoe_status zmoe_ep_create(const zmoe_ep_config* cfg, zmoe_layer* local, zmoe_ep** out);
zmoe_status zmoe_ep_destroy(zmoe_ep* ep);
/* Host pointers, copied to HBM.  bias ([E] fp32) and w_shared_gate ([H] BF16) may be NULL. */
zmoe_status zmoe_ep_set_router(zmoe_ep* ep, const uint16_t* w_router, const float* bias,
                               const uint16_t* w_shared_gate);
zmoe_status zmoe_ep_set_shared(zmoe_ep* ep, const uint16_t* gate, const uint16_t* up, const uint16_t* down);
/* x, out: device [T, H] BF16, T <= max_tokens (T = 0 still takes part in the exchanges). */
zmoe_status zmoe_ep_forward(zmoe_ep* ep, const uint16_t* x, int T, uint16_t* out, zmoe_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* ZMOE_H_ */
