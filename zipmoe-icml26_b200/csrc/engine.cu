// MoE-layer engine: HBM-resident compressed expert store, decoded-expert
// cache, on-demand decode of misses, and the layer forward
// router -> permute -> decode misses -> grouped FFN (+ shared expert) -> combine.
//
// Re-targets the reference's host runtime for one layer:
//  * TensorEngine::ToWorkers / ZipMoESchedulerFunc (csrc/tensor_engine/tensor_engine.cpp:515-669)
//    and its CPU LZ4 workers: misses become one fused decode launch over all
//    their chunks, reading LZ4 blocks that already sit in HBM;
//  * ZipMoECacheHandle::ProactiveDecision and the slot policies
//    (csrc/memory/cache.cpp:226-270, :445-690): NORMAL -> decode into a cache
//    slot (evicting a victim that this forward does not use), EVICT -> decode
//    into a transient slot that is reused by the next forward;
//  * ExpertDispatcher's fetch/exec/output threads (csrc/dispatcher/expert_dispatcher.cpp:285-499):
//    one stream-ordered launch sequence, with one host synchronisation to read
//    the per-expert token counts (the reference's expert_count.cpu(),
//    experts/expert_executor.py:45-49).
#include <algorithm>
#include <deque>
#include <memory>
#include <numeric>
#include <vector>

#include "common.cuh"

namespace zmoe {

zmoe_status launch_decode_chunks(const zmoe_chunk*, int, int32_t*, cudaStream_t);
zmoe_status launch_router(const zmoe_router_args*, cudaStream_t);
zmoe_status launch_permute(const zmoe_permute_args*, cudaStream_t);
zmoe_status launch_combine(const zmoe_combine_args*, cudaStream_t);

namespace {

struct TensorStore {
  // [LZ4 blocks, each 16-byte aligned][sign+mantissa plane][segment indexes],
  // in device memory, or in pinned host memory for a host-tier layer
  uint8_t* dev = nullptr;
  uint8_t* host = nullptr;
  bool loaded() const { return dev || host; }
  std::vector<uint32_t> block_off, block_size, orig_size;
  std::vector<uint64_t> idx_off;   // byte offset of each block's index
  std::vector<uint32_t> idx_n;     // entries of each block's index
  uint64_t sm_off = 0, numel = 0, bytes = 0;
};

constexpr uint32_t kSegBytes = ZMOE_SLICE_BYTES;

template <class T>
T* dmalloc(size_t n, zmoe_status* st) {
  void* p = nullptr;
  if (n == 0) n = 1;
  if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
    set_error("cudaMalloc of %zu bytes failed", n * sizeof(T));
    *st = ZMOE_ENOMEM;
    return nullptr;
  }
  return static_cast<T*>(p);
}

template <class T>
T* hmalloc(size_t n, zmoe_status* st) {
  void* p = nullptr;
  if (n == 0) n = 1;
  if (cudaMallocHost(&p, n * sizeof(T)) != cudaSuccess) {
    set_error("cudaMallocHost of %zu bytes failed", n * sizeof(T));
    *st = ZMOE_ENOMEM;
    return nullptr;
  }
  return static_cast<T*>(p);
}

}  // namespace

struct Layer {
  zmoe_layer_config cfg{};
  int tensors = 3;                 // per expert: 3 (SwiGLU) or 2 (ReLU)
  uint64_t numel = 0;              // elements per expert tensor (H * I)
  std::vector<std::vector<TensorStore>> store;   // [E][tensors]

  // decoded slots: cache slots first, then transient slots
  uint16_t* slots = nullptr;
  int n_cache = 0, n_transient = 0;
  std::vector<int> slot_owner;     // expert or -1
  std::vector<int> expert_slot;    // slot or -1 (cache slots only)
  std::vector<uint64_t> slot_count, slot_stamp, slot_admit;
  std::vector<uint64_t> global_count;
  uint64_t clock = 0;

  // weights owned by the layer
  uint16_t* w_router = nullptr;
  float* bias = nullptr;
  uint16_t* w_sgate = nullptr;
  uint16_t* w_shared[3] = {nullptr, nullptr, nullptr};

  // workspace
  int max_rows = 0;
  int32_t *idx = nullptr, *counts = nullptr, *offsets = nullptr, *row_of = nullptr, *tor = nullptr;
  float *tw = nullptr, *sg = nullptr;
  uint16_t *y = nullptr, *ysh = nullptr;              // BF16 expert rows
  uint16_t *xp = nullptr, *h = nullptr, *hsh = nullptr;
  zmoe_chunk* desc_dev = nullptr;
  int32_t* status_dev = nullptr;
  const uint16_t** wtab_dev = nullptr;
  int32_t* counts_host = nullptr;
  int32_t* offsets_host = nullptr;     // zmoe_layer_experts: group offsets staged for upload
  int32_t* offsets_ext = nullptr;      // ... and on the device
  zmoe_chunk* desc_host = nullptr;
  const uint16_t** wtab_host = nullptr;
  int32_t* status_host = nullptr;
  int max_desc = 0, max_waves = 0;
  // The pinned descriptor / status buffers (desc_host, status_host) and their
  // device twins are used as a ring: each decode takes the next count entries
  // and keeps them until the copy of its status words has landed.
  int desc_cursor = 0;
  struct PendingDecode { int base, count; cudaEvent_t done; };
  std::deque<PendingDecode> pending;
  std::vector<cudaEvent_t> free_events;
  zmoe_status reclaim(bool wait_all);
  zmoe_status alloc_desc(int count, int* base);
  // Misses decode on the layer's own stream (the device's highest priority),
  // while the caller's stream runs the FFN over cache hits and the shared
  // expert; events order the two where slots are shared.
  cudaStream_t ds = nullptr;
  cudaEvent_t ev_caller = nullptr;      // caller's stream -> decode stream
  cudaEvent_t ev_decoded = nullptr;     // decode stream -> caller's stream
  cudaEvent_t ev_prefetch = nullptr;    // end of the last prefetch decode
  bool prefetch_pending = false;
  uint32_t* map_scratch = nullptr; // decoder source-map scratch (zmoe_decode_scratch_bytes per chunk)
  bool host_store = false;         // compressed experts in pinned host memory, copied in per miss
  // host tier: pool of sign+mantissa planes kept in HBM (SMCACHE experts)
  int n_sm = 0;
  uint8_t* sm_pool = nullptr;      // n_sm * tensors * numel bytes
  std::vector<int> sm_owner, expert_sm;
  std::vector<uint64_t> sm_stamp;
  std::vector<char> sm_fill;       // this forward: planes to copy into the pool before decoding
  uint8_t* sm_plane(int e, int t) const { return sm_pool + ((size_t)expert_sm[e] * tensors + t) * numel; }
  int choose_sm_victim(const std::vector<char>& active);
  uint8_t* stage_buf = nullptr;    // host tier: device copies of the compressed tensors being decoded
  uint64_t stage_cap = 0;
  uint64_t map_cap = 0;            // bytes of map_scratch
  // error word of this layer's FFN launches (set when a bounded wait ran out),
  // copied back after each call and checked at the next one
  int32_t* kerr_dev = nullptr;
  int32_t* kerr_host = nullptr;
  cudaEvent_t kerr_ready = nullptr;
  bool kerr_pending = false;
  zmoe_status queue_kernel_error_copy(cudaStream_t s);
  zmoe_status check_kernel_error(bool wait);
  // host-side pass-through buffers for forward_host
  uint16_t* x_stage = nullptr;
  uint16_t* out_stage = nullptr;
  // submit_host: two staging slots, copies on their own streams
  uint16_t* x_slot[2] = {nullptr, nullptr};
  uint16_t* out_slot[2] = {nullptr, nullptr};
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t in_done[2] = {nullptr, nullptr}, fwd_done[2] = {nullptr, nullptr}, out_done[2] = {nullptr, nullptr};
  uint64_t submitted = 0;
  zmoe_status submit_host(const uint16_t* x_host, int T, uint16_t* out_host, cudaStream_t s);
  cudaEvent_t offsets_ready = nullptr;   // zmoe_layer_experts: the pinned offsets were copied
  cudaEvent_t counts_ready = nullptr;    // forward: the per-expert counts reached the host
  bool offsets_pending = false;

  // optional per-kernel timing: events around decode and FFN launches on the
  // launch stream, folded into stats at the next synchronisation
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  struct Timed { int ev; int kind; uint64_t bytes; };   // events ev (start), ev + 1 (stop)
  std::vector<Timed> ev_pending;
  int ev_used = 0;
  cudaEvent_t next_event();
  zmoe_status fold_timing();

  zmoe_layer_stats stats{};

  ~Layer();
  zmoe_status init(const zmoe_layer_config& c);
  zmoe_status forward(const uint16_t* x, int T, uint16_t* out, cudaStream_t s);
  zmoe_status run_experts(const uint16_t* xrows, const int32_t* offsets_dev, const int32_t* counts_h, int rows,
                          uint16_t* yrows, cudaStream_t s, bool caller_marked);
  zmoe_status experts(const uint16_t* xrows, const int32_t* counts_h, int rows, uint16_t* yrows, cudaStream_t s);
  zmoe_status check_status();
  int choose_victim(const std::vector<char>& active);
  // defer_status: the copy of the chunks' status words to the host waits for
  // queue_status, so that work queued meanwhile (the FFN over the decoded
  // experts) follows the decode directly on the stream
  zmoe_status decode_into(const std::vector<std::pair<int, int>>& jobs, cudaStream_t s, bool defer_status = false);
  zmoe_status queue_status(cudaStream_t s);
  std::vector<std::pair<int, int>> status_deferred;   // (base, count) of decodes whose status copy waits
  zmoe_status ffn_over(const std::vector<std::pair<int, int>>& groups, int table, const uint16_t* xrows,
                       const int32_t* offsets_dev, int rows, uint16_t* yrows, cudaStream_t s);
  uint16_t* slot_ptr(int slot, int t) const { return slots + ((size_t)slot * tensors + t) * numel; }
};

Layer::~Layer() {
  for (auto& e : store)
    for (auto& t : e) { cudaFree(t.dev); cudaFreeHost(t.host); }
  cudaFree(stage_buf);
  cudaFree(sm_pool);
  cudaFree(slots);
  cudaFree(w_router); cudaFree(bias); cudaFree(w_sgate);
  for (auto* p : w_shared) cudaFree(p);
  cudaFree(idx); cudaFree(counts); cudaFree(offsets); cudaFree(row_of); cudaFree(tor);
  cudaFree(tw); cudaFree(sg); cudaFree(y); cudaFree(ysh); cudaFree(xp); cudaFree(h); cudaFree(hsh);
  cudaFree(desc_dev); cudaFree(status_dev); cudaFree(wtab_dev);
  cudaFree(offsets_ext); cudaFreeHost(offsets_host);
  cudaFreeHost(counts_host); cudaFreeHost(desc_host); cudaFreeHost(wtab_host); cudaFreeHost(status_host);
  cudaFree(x_stage); cudaFree(out_stage); cudaFree(map_scratch);
  cudaFree(kerr_dev); cudaFreeHost(kerr_host);
  if (kerr_ready) cudaEventDestroy(kerr_ready);
  cudaFree(x_slot[1]); cudaFree(out_slot[1]);          // slot 0 is x_stage / out_stage
  for (int i = 0; i < 2; ++i)
    for (cudaEvent_t e : {in_done[i], fwd_done[i], out_done[i]})
      if (e) cudaEventDestroy(e);
  if (copy_in) cudaStreamDestroy(copy_in);
  if (copy_out) cudaStreamDestroy(copy_out);
  for (auto& p : pending) cudaEventDestroy(p.done);
  for (auto e : free_events) cudaEventDestroy(e);
  for (cudaEvent_t e : {ev_caller, ev_decoded, ev_prefetch})
    if (e) cudaEventDestroy(e);
  if (ds) cudaStreamDestroy(ds);
  if (offsets_ready) cudaEventDestroy(offsets_ready);
  if (counts_ready) cudaEventDestroy(counts_ready);
  for (auto e : ev_pool) cudaEventDestroy(e);
}

cudaEvent_t Layer::next_event() {
  if (ev_used == (int)ev_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    ev_pool.push_back(e);
  }
  return ev_pool[ev_used++];
}

zmoe_status Layer::fold_timing() {
  for (const Timed& t : ev_pending) {
    float ms = 0.f;
    ZMOE_CUDA_RET(cudaEventSynchronize(ev_pool[t.ev + 1]));
    ZMOE_CUDA_RET(cudaEventElapsedTime(&ms, ev_pool[t.ev], ev_pool[t.ev + 1]));
    const uint64_t ns = (uint64_t)((double)ms * 1.0e6);
    if (t.kind == 0) {
      stats.decode_ns += ns;
      stats.decode_timed_bytes += t.bytes;
      stats.decode_timed_launches++;
    } else {
      stats.ffn_ns += ns;
      stats.ffn_timed_launches++;
    }
  }
  ev_pending.clear();
  ev_used = 0;
  return ZMOE_OK;
}

zmoe_status Layer::init(const zmoe_layer_config& c) {
  cfg = c;
  ZMOE_CHECK_ARG(c.hidden > 0 && c.hidden % 256 == 0, "layer: hidden=%d must be a positive multiple of 256", c.hidden);
  ZMOE_CHECK_ARG(c.inter > 0 && c.inter % 8 == 0, "layer: inter=%d must be a positive multiple of 8", c.inter);
  ZMOE_CHECK_ARG(c.num_experts >= 1 && c.num_experts <= 256, "layer: num_experts=%d outside [1, 256]", c.num_experts);
  ZMOE_CHECK_ARG(c.topk >= 1 && c.topk <= 8 && c.topk <= c.num_experts, "layer: bad topk=%d", c.topk);
  ZMOE_CHECK_ARG(c.kind == 0 || c.kind == 1, "layer: kind must be 0 (SwiGLU) or 1 (ReLU)");
  ZMOE_CHECK_ARG(c.route_mode >= 0 && c.route_mode <= 2, "layer: bad route_mode");
  ZMOE_CHECK_ARG(c.max_tokens >= 1, "layer: max_tokens must be >= 1");
  ZMOE_CHECK_ARG(c.cache_slots >= 0 && c.cache_slots <= c.num_experts, "layer: cache_slots outside [0, E]");
  ZMOE_CHECK_ARG(c.shared_inter == 0 || c.shared_inter % 8 == 0, "layer: shared_inter must be a multiple of 8");
  ZMOE_CHECK_ARG(c.route_mode != ZMOE_ROUTE_SWITCH || c.kind == 1, "layer: Switch routing needs ReLU experts");
  ZMOE_CHECK_ARG(c.sm_slots >= 0 && c.sm_slots <= c.num_experts, "layer: sm_slots outside [0, E]");
  tensors = c.kind == 0 ? 3 : 2;
  numel = (uint64_t)c.hidden * c.inter;
  const int E = c.num_experts;
  store.assign(E, std::vector<TensorStore>(tensors));
  n_cache = c.cache_slots;
  n_transient = c.transient_slots > 0 ? std::min(c.transient_slots, E) : E - n_cache;
  if (n_transient < 1) n_transient = 1;
  const int n_slots = n_cache + n_transient;
  slot_owner.assign(n_slots, -1);
  expert_slot.assign(E, -1);
  slot_count.assign(n_slots, 0);
  slot_stamp.assign(n_slots, 0);
  slot_admit.assign(n_slots, 0);
  global_count.assign(E, 0);
  expert_sm.assign(E, -1);
  sm_fill.assign(E, 0);
  zmoe_status st = ZMOE_OK;
  slots = dmalloc<uint16_t>((size_t)n_slots * tensors * numel, &st);
  const int T = c.max_tokens, k = c.topk, H = c.hidden;
  max_rows = T * k;
  idx = dmalloc<int32_t>((size_t)T * k, &st);
  tw = dmalloc<float>((size_t)T * k, &st);
  sg = dmalloc<float>(T, &st);
  counts = dmalloc<int32_t>(E, &st);
  offsets = dmalloc<int32_t>(E + 1, &st);
  row_of = dmalloc<int32_t>((size_t)T * k, &st);
  tor = dmalloc<int32_t>((size_t)T * k, &st);
  xp = dmalloc<uint16_t>((size_t)max_rows * H, &st);
  h = dmalloc<uint16_t>((size_t)max_rows * c.inter, &st);
  y = dmalloc<uint16_t>((size_t)max_rows * H, &st);
  if (c.shared_inter > 0) {
    ysh = dmalloc<uint16_t>((size_t)T * H, &st);
    hsh = dmalloc<uint16_t>((size_t)T * c.shared_inter, &st);
  }
  max_waves = (E + n_transient - 1) / n_transient + 1;
  max_desc = E * tensors * 64;
  desc_dev = dmalloc<zmoe_chunk>(max_desc, &st);
  status_dev = dmalloc<int32_t>(max_desc, &st);
  wtab_dev = dmalloc<const uint16_t*>((size_t)(max_waves + 1) * E * 3, &st);
  counts_host = hmalloc<int32_t>(E, &st);
  offsets_host = hmalloc<int32_t>(E + 1, &st);
  offsets_ext = dmalloc<int32_t>(E + 1, &st);
  desc_host = hmalloc<zmoe_chunk>(max_desc, &st);
  wtab_host = hmalloc<const uint16_t*>((size_t)(max_waves + 1) * E * 3, &st);
  status_host = hmalloc<int32_t>(max_desc, &st);
  x_stage = dmalloc<uint16_t>((size_t)T * H, &st);
  out_stage = dmalloc<uint16_t>((size_t)T * H, &st);
  x_slot[0] = x_stage;
  out_slot[0] = out_stage;
  x_slot[1] = dmalloc<uint16_t>((size_t)T * H, &st);
  out_slot[1] = dmalloc<uint16_t>((size_t)T * H, &st);
  kerr_dev = dmalloc<int32_t>(1, &st);
  kerr_host = hmalloc<int32_t>(1, &st);
  if (st != ZMOE_OK) return st;
  ZMOE_CUDA_RET(cudaMemset(kerr_dev, 0, sizeof(int32_t)));
  *kerr_host = 0;
  memset(counts_host, 0, sizeof(int32_t) * E);
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&kerr_ready, cudaEventDisableTiming));
  ZMOE_CUDA_RET(cudaStreamCreateWithFlags(&copy_in, cudaStreamNonBlocking));
  ZMOE_CUDA_RET(cudaStreamCreateWithFlags(&copy_out, cudaStreamNonBlocking));
  for (int i = 0; i < 2; ++i) {
    ZMOE_CUDA_RET(cudaEventCreateWithFlags(&in_done[i], cudaEventDisableTiming));
    ZMOE_CUDA_RET(cudaEventCreateWithFlags(&fwd_done[i], cudaEventDisableTiming));
    ZMOE_CUDA_RET(cudaEventCreateWithFlags(&out_done[i], cudaEventDisableTiming));
  }
  int least = 0, greatest = 0;
  ZMOE_CUDA_RET(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  ZMOE_CUDA_RET(cudaStreamCreateWithPriority(&ds, cudaStreamNonBlocking, greatest));
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&ev_caller, cudaEventDisableTiming));
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&ev_decoded, cudaEventDisableTiming));
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&ev_prefetch, cudaEventDisableTiming));
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&offsets_ready, cudaEventDisableTiming));
  ZMOE_CUDA_RET(cudaEventCreateWithFlags(&counts_ready, cudaEventDisableTiming));
  return ZMOE_OK;
}

// A pool slot for a sign+mantissa plane: a free one, else the least recently
// used plane of an expert this forward does not use.
int Layer::choose_sm_victim(const std::vector<char>& active) {
  int victim = -1;
  uint64_t best = UINT64_MAX;
  for (int s = 0; s < n_sm; ++s) {
    const int e = sm_owner[s];
    if (e < 0) return s;
    if (active[e] || sm_fill[e]) continue;
    if (sm_stamp[s] < best) { best = sm_stamp[s]; victim = s; }
  }
  return victim;
}

int Layer::choose_victim(const std::vector<char>& active) {
  int victim = -1;
  uint64_t best = UINT64_MAX;
  for (int s = 0; s < n_cache; ++s) {
    const int e = slot_owner[s];
    if (e < 0) return s;                      // free slot
    if (active[e]) continue;                  // protected: used by this forward
    uint64_t key;
    switch (cfg.cache_policy) {
      case ZMOE_CACHE_LRU: key = slot_stamp[s]; break;
      case ZMOE_CACHE_FIFO: key = slot_admit[s]; break;
      case ZMOE_CACHE_LFU: key = global_count[e]; break;
      default: key = slot_count[s]; break;     // ZipMoE: tokens served since admission
    }
    if (key < best) { best = key; victim = s; }
  }
  return victim;
}

// Checks the status words of every decode whose status copy has landed (all
// of them with wait_all) and frees their ring entries.  Returns the first
// decode error found.
zmoe_status Layer::reclaim(bool wait_all) {
  zmoe_status bad = ZMOE_OK;
  while (!pending.empty()) {
    PendingDecode p = pending.front();
    if (wait_all) {
      ZMOE_CUDA_RET(cudaEventSynchronize(p.done));
    } else {
      const cudaError_t q = cudaEventQuery(p.done);
      if (q == cudaErrorNotReady) break;
      ZMOE_CUDA_RET(q);
    }
    for (int i = 0; i < p.count && bad == ZMOE_OK; ++i) {
      if (status_host[p.base + i] != ZMOE_CHUNK_OK) {
        stats.decode_errors++;
        set_error("decode of chunk %d failed with status %d", i, status_host[p.base + i]);
        bad = ZMOE_EINVAL;
      }
    }
    free_events.push_back(p.done);
    pending.pop_front();
  }
  if (pending.empty()) desc_cursor = 0;
  return bad;
}

zmoe_status Layer::check_status() { return reclaim(false); }

zmoe_status Layer::alloc_desc(int count, int* base) {
  ZMOE_CHECK_ARG(count <= max_desc, "too many chunks in one decode (%d > %d)", count, max_desc);
  zmoe_status st = reclaim(false);
  if (st != ZMOE_OK) return st;
  if (desc_cursor + count > max_desc && (st = reclaim(true)) != ZMOE_OK) return st;
  *base = desc_cursor;
  desc_cursor += count;
  return ZMOE_OK;
}

// After a call's FFN launches: copy the error word back (unless the previous
// copy is still unread; the word stays set until it is reported, so that copy
// or a later one sees it).
zmoe_status Layer::queue_kernel_error_copy(cudaStream_t s) {
  if (kerr_pending) return ZMOE_OK;
  ZMOE_CUDA_RET(cudaMemcpyAsync(kerr_host, kerr_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  ZMOE_CUDA_RET(cudaEventRecord(kerr_ready, s));
  kerr_pending = true;
  return ZMOE_OK;
}

// Reports (once) an FFN launch that gave up a bounded wait.  Without wait, a
// copy that has not landed yet is left for the next check.
zmoe_status Layer::check_kernel_error(bool wait) {
  if (!kerr_pending) return ZMOE_OK;
  if (wait) {
    ZMOE_CUDA_RET(cudaEventSynchronize(kerr_ready));
  } else {
    const cudaError_t q = cudaEventQuery(kerr_ready);
    if (q == cudaErrorNotReady) return ZMOE_OK;
    ZMOE_CUDA_RET(q);
  }
  kerr_pending = false;
  if (*kerr_host != 0) {
    const int32_t code = *kerr_host;
    *kerr_host = 0;
    ZMOE_CUDA_RET(cudaMemset(kerr_dev, 0, sizeof(int32_t)));
    set_error("an expert FFN launch of an earlier call gave up a bounded wait (code %d); its outputs are "
              "incomplete", code);
    return ZMOE_EKERNEL;
  }
  return ZMOE_OK;
}

// Decode (expert, slot) jobs in one fused launch on stream s (the decode stream).
zmoe_status Layer::decode_into(const std::vector<std::pair<int, int>>& jobs, cudaStream_t s, bool defer_status) {
  int cnt = 0;
  for (auto [e, slot] : jobs)
    for (int t = 0; t < tensors; ++t) cnt += (int)store[e][t].block_off.size();
  if (cnt == 0) return ZMOE_OK;
  int base = 0;
  // a status copy still deferred (an earlier call stopped on an error) is
  // queued first, so that descriptor reuse sees every decode in flight
  zmoe_status st = status_deferred.empty() ? ZMOE_OK : queue_status(s);
  if (st != ZMOE_OK) return st;
  st = alloc_desc(cnt, &base);
  if (st != ZMOE_OK) return st;
  // host tier: each tensor's packed buffer is copied into the staging area
  // ahead of the decode (stream order keeps the previous decode's reads of the
  // area before these copies)
  if (host_store) {
    uint64_t need = 0;
    for (auto [e, slot] : jobs)
      for (int t = 0; t < tensors; ++t) need += store[e][t].bytes;    // an upper bound with resident planes
    if (need > stage_cap) {
      ZMOE_CUDA_RET(cudaStreamSynchronize(s));
      cudaFree(stage_buf);
      stage_buf = nullptr;
      stage_cap = 0;
      ZMOE_CUDA_RET(cudaMalloc(&stage_buf, need));
      stage_cap = need;
    }
  }
  uint64_t stage_off = 0;
  int nd = base;
  for (auto [e, slot] : jobs) {
    for (int t = 0; t < tensors; ++t) {
      const TensorStore& ts = store[e][t];
      const uint8_t* buf = ts.dev;
      const uint8_t* smbase = nullptr;                 // the plane, when not in buf at sm_off
      uint64_t idx_shift = 0;                          // the indexes sit this much lower in the staged copy
      if (host_store) {
        uint8_t* at = stage_buf + stage_off;           // offsets stay 16-byte aligned (bytes is)
        const bool resident = n_sm > 0 && expert_sm[e] >= 0;
        if (resident) {
          // blocks, then indexes; the plane comes from the pool (copied in first when new)
          if (sm_fill[e]) {
            ZMOE_CUDA_RET(cudaMemcpyAsync(sm_plane(e, t), ts.host + ts.sm_off, ts.numel, cudaMemcpyHostToDevice,
                                          s));
            stats.host_copy_bytes += ts.numel;
          }
          const uint64_t idx0 = ts.idx_off.empty() ? ts.bytes : ts.idx_off[0];
          ZMOE_CUDA_RET(cudaMemcpyAsync(at, ts.host, ts.sm_off, cudaMemcpyHostToDevice, s));
          ZMOE_CUDA_RET(cudaMemcpyAsync(at + ts.sm_off, ts.host + idx0, ts.bytes - idx0, cudaMemcpyHostToDevice, s));
          stats.host_copy_bytes += ts.sm_off + (ts.bytes - idx0);
          stats.sm_resident_tensors++;
          stage_off += ts.sm_off + (ts.bytes - idx0);
          smbase = sm_plane(e, t);
          idx_shift = idx0 - ts.sm_off;
        } else {
          ZMOE_CUDA_RET(cudaMemcpyAsync(at, ts.host, ts.bytes, cudaMemcpyHostToDevice, s));
          stats.host_copy_bytes += ts.bytes;
          stage_off += ts.bytes;
        }
        buf = at;
      }
      uint64_t e0 = 0;
      uint16_t* dst = slot_ptr(slot, t);
      for (size_t c = 0; c < ts.block_off.size(); ++c) {
        zmoe_chunk& d = desc_host[nd++];
        d.src = buf + ts.block_off[c];
        d.sm = (smbase ? smbase : buf + ts.sm_off) + e0;
        d.dst = dst + e0;
        d.src_size = ts.block_size[c];
        d.out_size = ts.orig_size[c];
        d.index = reinterpret_cast<const uint32_t*>(buf + ts.idx_off[c] - idx_shift);
        d.n_index = ts.idx_n[c];
        d.seg_bytes = kSegBytes;
        d.map = nullptr;                     // assigned below, one scratch area per chunk
        stats.decoded_bytes += (uint64_t)ts.block_size[c] + 3ull * ts.orig_size[c];
        e0 += ts.orig_size[c];
      }
    }
    stats.decoded_experts++;
  }
  uint64_t need = 0;
  for (int i = 0; i < cnt; ++i) need += zmoe_decode_scratch_bytes(desc_host[base + i].out_size);
  if (need > map_cap) {
    // grows to the largest decode seen (a synchronising allocation, only
    // before the working set is known); every decode runs on this stream
    ZMOE_CUDA_RET(cudaStreamSynchronize(s));
    cudaFree(map_scratch);
    map_scratch = nullptr;
    map_cap = 0;
    ZMOE_CUDA_RET(cudaMalloc(&map_scratch, need));
    map_cap = need;
  }
  uint64_t moff = 0;
  for (int i = 0; i < cnt; ++i) {
    desc_host[base + i].map = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(map_scratch) + moff);
    moff += zmoe_decode_scratch_bytes(desc_host[base + i].out_size);
  }
  ZMOE_CUDA_RET(cudaMemcpyAsync(desc_dev + base, desc_host + base, sizeof(zmoe_chunk) * cnt,
                                cudaMemcpyHostToDevice, s));
  uint64_t bytes = 0;
  for (int i = base; i < nd; ++i) bytes += (uint64_t)desc_host[i].src_size + 3ull * desc_host[i].out_size;
  int ev = -1;
  if (timing) {
    ev = ev_used;
    cudaEvent_t a = next_event(), b = next_event();
    if (!a || !b) { set_error("cudaEventCreate failed"); return ZMOE_ECUDA; }
    ZMOE_CUDA_RET(cudaEventRecord(a, s));
  }
  st = launch_decode_chunks(desc_dev + base, cnt, status_dev + base, s);
  if (st != ZMOE_OK) return st;
  if (timing) {
    ZMOE_CUDA_RET(cudaEventRecord(ev_pool[ev + 1], s));
    ev_pending.push_back({ev, 0, bytes});
  }
  stats.launches += 2;                        // map_kernel + resolve_kernel
  stats.decode_launches++;
  stats.decoded_chunks += cnt;
  status_deferred.push_back({base, cnt});
  return defer_status ? ZMOE_OK : queue_status(s);
}

// Copies the status words of the deferred decodes to the host on stream s and
// records when they have landed (checked at the next sync point).
zmoe_status Layer::queue_status(cudaStream_t s) {
  for (auto [base, cnt] : status_deferred) {
    ZMOE_CUDA_RET(cudaMemcpyAsync(status_host + base, status_dev + base, sizeof(int32_t) * cnt,
                                  cudaMemcpyDeviceToHost, s));
    cudaEvent_t done = nullptr;
    if (!free_events.empty()) {
      done = free_events.back();
      free_events.pop_back();
    } else {
      ZMOE_CUDA_RET(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    }
    ZMOE_CUDA_RET(cudaEventRecord(done, s));
    pending.push_back({base, cnt, done});
  }
  status_deferred.clear();
  return ZMOE_OK;
}

// Grouped FFN over the given (expert, slot) groups on stream s; the other
// groups of the launch are skipped.  table: which host weight table to fill.
zmoe_status Layer::ffn_over(const std::vector<std::pair<int, int>>& groups, int table, const uint16_t* xrows,
                            const int32_t* offsets_dev, int rows, uint16_t* yrows, cudaStream_t s) {
  if (groups.empty()) return ZMOE_OK;
  const int E = cfg.num_experts;
  if (table > max_waves) { set_error("too many decode waves"); return ZMOE_EUNSUPPORTED; }
  const uint16_t** tab = wtab_host + (size_t)table * E * 3;
  std::fill(tab, tab + (size_t)E * 3, nullptr);
  for (auto [e, slot] : groups) {
    tab[e * 3 + 0] = slot_ptr(slot, 0);
    tab[e * 3 + 1] = tensors == 3 ? slot_ptr(slot, 1) : nullptr;
    tab[e * 3 + 2] = slot_ptr(slot, tensors - 1);
  }
  zmoe_ffn_args fa{};
  fa.x = xrows; fa.w = tab; fa.offsets = offsets_dev; fa.G = E; fa.rows_total = rows; fa.H = cfg.hidden;
  fa.I = cfg.inter; fa.kind = cfg.kind; fa.h = h; fa.y = yrows;
  int ev = -1;
  if (timing) {
    ev = ev_used;
    cudaEvent_t a = next_event(), b = next_event();
    if (!a || !b) { set_error("cudaEventCreate failed"); return ZMOE_ECUDA; }
    ZMOE_CUDA_RET(cudaEventRecord(a, s));
  }
  zmoe_status st = launch_expert_ffn(&fa, s, kerr_dev);
  if (st != ZMOE_OK) return st;
  if (timing) {
    ZMOE_CUDA_RET(cudaEventRecord(ev_pool[ev + 1], s));
    ev_pending.push_back({ev, 1, 0});
  }
  stats.launches += 2;
  return ZMOE_OK;
}

// Cache decisions (ProactiveDecision), miss decode waves and the grouped FFN
// over rows already grouped by expert: group e is rows [offsets[e], offsets[e+1]).
// caller_marked: ev_caller was recorded on s before any work of this call
// (otherwise it is recorded here).
zmoe_status Layer::run_experts(const uint16_t* xrows, const int32_t* offsets_dev, const int32_t* counts_h, int rows,
                               uint16_t* yrows, cudaStream_t s, bool caller_marked) {
  const int E = cfg.num_experts;
  zmoe_status st;
  // 3. cache decisions (ProactiveDecision)
  std::vector<char> active(E, 0);
  std::vector<int> act;
  for (int e = 0; e < E; ++e)
    if (counts_h[e] > 0) { active[e] = 1; act.push_back(e); global_count[e] += counts_h[e]; }
  ++clock;
  std::vector<int> ranked(act);
  std::vector<std::pair<int, int>> hits_slots;       // (expert, slot) ready to use
  std::vector<int> misses;
  for (int e : act) {
    const int sl = expert_slot[e];
    if (sl >= 0) {
      stats.hits++;
      slot_count[sl] += counts_h[e];
      slot_stamp[sl] = clock;
      hits_slots.push_back({e, sl});
    } else {
      stats.misses++;
      misses.push_back(e);
    }
  }
  // rank of each miss by global count (count_up of cache.cpp:230-238)
  std::vector<std::pair<int, int>> to_cache, to_transient;
  const double thr_normal = n_cache + cfg.state_margin * E;
  const double thr_sm = n_cache + n_sm + cfg.state_margin * E;   // Threshold_SMCACHE (cache.cpp:122-123)
  std::fill(sm_fill.begin(), sm_fill.end(), 0);
  for (int e : misses) {
    int up = 0;
    for (int q = 0; q < E; ++q) up += global_count[q] > global_count[e];
    int slot = -1;
    if (n_cache > 0 && up < thr_normal) {
      slot = choose_victim(active);
      if (slot >= 0) {
        if (slot_owner[slot] >= 0) { expert_slot[slot_owner[slot]] = -1; stats.evictions++; }
        slot_owner[slot] = e;
        expert_slot[e] = slot;
        slot_count[slot] = counts_h[e];
        slot_stamp[slot] = clock;
        slot_admit[slot] = clock;
        to_cache.push_back({e, slot});
        continue;
      }
    }
    to_transient.push_back({e, -1});
    // SMCACHE: not decoded-cached, but ranked high enough to keep its planes in HBM
    if (n_sm > 0 && up < thr_sm) {
      if (expert_sm[e] < 0) {
        const int ps = choose_sm_victim(active);
        if (ps >= 0) {
          if (sm_owner[ps] >= 0) expert_sm[sm_owner[ps]] = -1;
          sm_owner[ps] = e;
          expert_sm[e] = ps;
          sm_fill[e] = 1;
        }
      }
      if (expert_sm[e] >= 0) sm_stamp[expert_sm[e]] = clock;
    }
  }

  // 4. Misses decode on the decode stream, in waves of the transient slots;
  //    the FFN over the cache hits runs on the caller's stream meanwhile, and
  //    the FFN over each decoded wave follows its decode.  Every slot a decode
  //    overwrites was last read by FFN work queued on s before ev_caller or
  //    earlier on the decode stream.
  if (!caller_marked) ZMOE_CUDA_RET(cudaEventRecord(ev_caller, s));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(ds, ev_caller, 0));
  size_t tpos = 0;
  int table = 0;
  std::vector<std::pair<int, int>> jobs(to_cache);
  auto next_wave = [&]() {
    int used = 0;
    while (tpos < to_transient.size() && used < n_transient) {
      jobs.push_back({to_transient[tpos].first, n_cache + used});
      ++tpos;
      ++used;
    }
  };
  next_wave();
  if ((st = decode_into(jobs, ds, true)) != ZMOE_OK) return st; // the critical path goes first
  if (!hits_slots.empty()) {
    if (prefetch_pending) {                                      // hits may sit in slots a prefetch filled
      ZMOE_CUDA_RET(cudaStreamWaitEvent(s, ev_prefetch, 0));
      prefetch_pending = false;
    }
    if ((st = ffn_over(hits_slots, table++, xrows, offsets_dev, rows, yrows, s)) != ZMOE_OK) return st;
  }
  // The FFN over each decoded wave follows its decode on the decode stream, so
  // it starts the moment the decode ends, beside what the caller's stream
  // still runs (the tail of the FFN over the hits); the next wave's decode,
  // which reuses the transient slots, follows that FFN on the same stream.
  // The two FFN launches write disjoint rows of h and yrows.
  while (!jobs.empty()) {
    if ((st = ffn_over(jobs, table++, xrows, offsets_dev, rows, yrows, ds)) != ZMOE_OK) return st;
    if ((st = queue_status(ds)) != ZMOE_OK) return st;
    jobs.clear();
    next_wave();
    if (jobs.empty()) break;
    if ((st = decode_into(jobs, ds, true)) != ZMOE_OK) return st;
  }
  if ((st = queue_status(ds)) != ZMOE_OK) return st;        // a decode with no FFN after it (none queued)
  ZMOE_CUDA_RET(cudaEventRecord(ev_decoded, ds));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(s, ev_decoded, 0));
  return ZMOE_OK;
}

// Expert stage alone, for callers that route and exchange rows themselves
// (expert parallelism): counts_h[e] rows of local expert e, grouped in order.
zmoe_status Layer::experts(const uint16_t* xrows, const int32_t* counts_h, int rows, uint16_t* yrows,
                           cudaStream_t s) {
  const int E = cfg.num_experts;
  ZMOE_CHECK_ARG(counts_h && (rows == 0 || (xrows && yrows)), "experts: null pointer");
  ZMOE_CHECK_ARG(rows >= 0 && rows <= max_rows, "experts: rows=%d outside [0, max_tokens*topk=%d]", rows, max_rows);
  long long sum = 0;
  for (int e = 0; e < E; ++e) {
    ZMOE_CHECK_ARG(counts_h[e] >= 0, "experts: negative count for expert %d", e);
    sum += counts_h[e];
  }
  ZMOE_CHECK_ARG(sum == rows, "experts: counts sum to %lld, rows=%d", sum, rows);
  for (int e = 0; e < E; ++e)
    for (int t = 0; t < tensors; ++t)
      ZMOE_CHECK_ARG(store[e][t].loaded(), "experts: expert %d tensor %d not loaded", e, t);
  zmoe_status st;
  // The pinned offsets buffer of the previous call is rewritten below: wait
  // for its copy (an event, not the stream, so that the caller's queued work,
  // an exchange or a gather, runs on while this call plans and launches).
  // Decode statuses that have landed are checked without waiting.
  if (offsets_pending) {
    ZMOE_CUDA_RET(cudaEventSynchronize(offsets_ready));
    offsets_pending = false;
  }
  if ((st = check_status()) != ZMOE_OK) return st;
  if ((st = check_kernel_error(false)) != ZMOE_OK) return st;
  if ((st = fold_timing()) != ZMOE_OK) return st;
  if (rows == 0) return ZMOE_OK;
  offsets_host[0] = 0;
  for (int e = 0; e < E; ++e) {
    offsets_host[e + 1] = offsets_host[e] + counts_h[e];
    counts_host[e] = counts_h[e];
  }
  ZMOE_CUDA_RET(cudaMemcpyAsync(offsets_ext, offsets_host, sizeof(int32_t) * (E + 1), cudaMemcpyHostToDevice, s));
  ZMOE_CUDA_RET(cudaEventRecord(offsets_ready, s));
  offsets_pending = true;
  if ((st = run_experts(xrows, offsets_ext, counts_host, rows, yrows, s, false)) != ZMOE_OK) return st;
  if ((st = queue_kernel_error_copy(s)) != ZMOE_OK) return st;
  stats.forwards++;
  stats.tokens += rows;
  return ZMOE_OK;
}

zmoe_status Layer::forward(const uint16_t* x, int T, uint16_t* out, cudaStream_t s) {
  ZMOE_CHECK_ARG(x && out, "forward: null pointer");
  ZMOE_CHECK_ARG(T >= 0 && T <= cfg.max_tokens, "forward: T=%d outside [0, max_tokens=%d]", T, cfg.max_tokens);
  ZMOE_CHECK_ARG(w_router, "forward: router weights not set");
  const int E = cfg.num_experts, k = cfg.topk, H = cfg.hidden;
  for (int e = 0; e < E; ++e)
    for (int t = 0; t < tensors; ++t)
      ZMOE_CHECK_ARG(store[e][t].loaded(), "forward: expert %d tensor %d not loaded", e, t);
  if (T == 0) return ZMOE_OK;
  zmoe_status st;
  // everything queued so far (the previous forward's FFN reads of the slots)
  // comes before this forward's decodes; the shared expert below does not
  ZMOE_CUDA_RET(cudaEventRecord(ev_caller, s));

  // 1. router
  zmoe_router_args ra{};
  ra.x = x; ra.w = w_router; ra.bias = bias; ra.w_shared_gate = w_sgate;
  ra.T = T; ra.H = H; ra.E = E; ra.k = k; ra.mode = cfg.route_mode;
  ra.norm_topk_prob = cfg.norm_topk_prob; ra.scaling = cfg.scaling;
  ra.logits = nullptr; ra.topk_idx = idx; ra.topk_w = tw; ra.shared_gate = w_sgate ? sg : nullptr;
  if ((st = launch_router(&ra, s)) != ZMOE_OK) return st;
  stats.launches++;

  // 2. permute + counts to the host
  zmoe_permute_args pa{};
  pa.topk_idx = idx; pa.x = x; pa.T = T; pa.H = H; pa.E = E; pa.k = k;
  pa.capacity = cfg.route_mode == ZMOE_ROUTE_SWITCH ? cfg.capacity : 0;
  pa.seq_len = cfg.seq_len > 0 ? cfg.seq_len : T;
  pa.counts = counts; pa.offsets = offsets; pa.row_of = row_of; pa.token_of_row = tor; pa.xp = xp;
  if ((st = launch_permute(&pa, s)) != ZMOE_OK) return st;
  stats.launches += 3;
  ZMOE_CUDA_RET(cudaMemcpyAsync(counts_host, counts, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, s));
  ZMOE_CUDA_RET(cudaEventRecord(counts_ready, s));

  // shared expert first: it needs no decoded weights, and it keeps the GPU
  // busy while the host waits for the counts and makes the cache decisions
  if (cfg.shared_inter > 0 && w_shared[0]) {
    zmoe_ffn_args fa{};
    const uint16_t* tab[3] = {w_shared[0], w_shared[1], w_shared[2]};   // host table
    fa.x = x; fa.w = tab; fa.offsets = nullptr; fa.G = 1; fa.rows_total = T; fa.H = H;
    fa.I = cfg.shared_inter; fa.kind = 0; fa.h = hsh; fa.y = ysh;
    if ((st = launch_expert_ffn(&fa, s, kerr_dev)) != ZMOE_OK) return st;
    stats.launches += 2;
  }
  // everything before the counts copy is done, the previous forward's decode
  // and pinned-buffer copies included
  ZMOE_CUDA_RET(cudaEventSynchronize(counts_ready));
  if ((st = check_status()) != ZMOE_OK) return st;   // previous forward's decode
  if ((st = check_kernel_error(true)) != ZMOE_OK) return st;   // its FFN launches (done by now)
  if ((st = fold_timing()) != ZMOE_OK) return st;

  if ((st = run_experts(xp, offsets, counts_host, T * k, y, s, true)) != ZMOE_OK) return st;

  // 5. combine
  zmoe_combine_args ca{};
  ca.y = y; ca.y_shared = (cfg.shared_inter > 0 && w_shared[0]) ? ysh : nullptr;
  ca.shared_gate = w_sgate ? sg : nullptr; ca.row_of = row_of; ca.topk_w = tw; ca.x = x;
  ca.T = T; ca.H = H; ca.k = k; ca.mode = cfg.route_mode; ca.out = out;
  if ((st = launch_combine(&ca, s)) != ZMOE_OK) return st;
  if ((st = queue_kernel_error_copy(s)) != ZMOE_OK) return st;
  stats.launches++;
  stats.forwards++;
  stats.tokens += T;
  return ZMOE_OK;
}

// One step with host buffers, pipelined: the input copy (copy_in) into staging
// slot k = step % 2, the forward on s, the output copy (copy_out) from slot k.
// Slot k's input is rewritten only after the forward of two steps ago has run
// (fwd_done), and its output only after that step's output copy (out_done),
// so the next step's input copy and this step's output copy overlap compute.
zmoe_status Layer::submit_host(const uint16_t* x_host, int T, uint16_t* out_host, cudaStream_t s) {
  const int k = (int)(submitted & 1);
  const size_t bytes = (size_t)T * cfg.hidden * 2;
  if (submitted >= 2) ZMOE_CUDA_RET(cudaStreamWaitEvent(copy_in, fwd_done[k], 0));
  ZMOE_CUDA_RET(cudaMemcpyAsync(x_slot[k], x_host, bytes, cudaMemcpyHostToDevice, copy_in));
  ZMOE_CUDA_RET(cudaEventRecord(in_done[k], copy_in));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(s, in_done[k], 0));
  if (submitted >= 2) ZMOE_CUDA_RET(cudaStreamWaitEvent(s, out_done[k], 0));
  zmoe_status st = forward(x_slot[k], T, out_slot[k], s);
  if (st != ZMOE_OK) return st;
  ZMOE_CUDA_RET(cudaEventRecord(fwd_done[k], s));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(copy_out, fwd_done[k], 0));
  ZMOE_CUDA_RET(cudaMemcpyAsync(out_host, out_slot[k], bytes, cudaMemcpyDeviceToHost, copy_out));
  ZMOE_CUDA_RET(cudaEventRecord(out_done[k], copy_out));
  ++submitted;
  return ZMOE_OK;
}

}  // namespace zmoe

using zmoe::Layer;

extern "C" {

zmoe_status zmoe_layer_create(const zmoe_layer_config* cfg, zmoe_layer** out) {
  ZMOE_CHECK_ARG(cfg && out, "layer_create: null pointer");
  auto* L = new Layer();
  zmoe_status st = L->init(*cfg);
  if (st != ZMOE_OK) {
    delete L;
    *out = nullptr;
    return st;
  }
  *out = reinterpret_cast<zmoe_layer*>(L);
  return ZMOE_OK;
}

zmoe_status zmoe_layer_destroy(zmoe_layer* layer) {
  delete reinterpret_cast<Layer*>(layer);
  return ZMOE_OK;
}

static zmoe_status upload(void** dst, const void* src, size_t bytes) {
  ZMOE_CUDA_RET(cudaMalloc(dst, bytes));
  ZMOE_CUDA_RET(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
  return ZMOE_OK;
}

zmoe_status zmoe_layer_set_router(zmoe_layer* layer, const uint16_t* w_router, const float* bias,
                                  const uint16_t* w_shared_gate) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && w_router, "set_router: null pointer");
  const size_t H = L->cfg.hidden, E = L->cfg.num_experts;
  cudaFree(L->w_router); cudaFree(L->bias); cudaFree(L->w_sgate);
  L->w_router = nullptr; L->bias = nullptr; L->w_sgate = nullptr;
  zmoe_status st = upload((void**)&L->w_router, w_router, E * H * 2);
  if (st == ZMOE_OK && bias) st = upload((void**)&L->bias, bias, E * 4);
  if (st == ZMOE_OK && w_shared_gate) st = upload((void**)&L->w_sgate, w_shared_gate, H * 2);
  return st;
}

zmoe_status zmoe_layer_set_shared(zmoe_layer* layer, const uint16_t* gate, const uint16_t* up,
                                  const uint16_t* down) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && gate && up && down, "set_shared: null pointer");
  ZMOE_CHECK_ARG(L->cfg.shared_inter > 0, "set_shared: layer has no shared expert");
  const size_t n = (size_t)L->cfg.hidden * L->cfg.shared_inter * 2;
  const uint16_t* src[3] = {gate, up, down};
  for (int i = 0; i < 3; ++i) {
    cudaFree(L->w_shared[i]);
    L->w_shared[i] = nullptr;
    zmoe_status st = upload((void**)&L->w_shared[i], src[i], n);
    if (st != ZMOE_OK) return st;
  }
  return ZMOE_OK;
}

zmoe_status zmoe_layer_load_expert(zmoe_layer* layer, int expert, int tensor, const uint8_t* const* blocks,
                                   const uint32_t* block_sizes, const uint32_t* original_sizes, int n_chunks,
                                   const uint8_t* sm, uint64_t numel) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && blocks && block_sizes && original_sizes && sm, "load_expert: null pointer");
  ZMOE_CHECK_ARG(expert >= 0 && expert < L->cfg.num_experts, "load_expert: expert %d out of range", expert);
  ZMOE_CHECK_ARG(tensor >= 0 && tensor < L->tensors, "load_expert: tensor %d out of range", tensor);
  ZMOE_CHECK_ARG(numel == L->numel, "load_expert: numel %llu != H*I = %llu", (unsigned long long)numel,
                 (unsigned long long)L->numel);
  ZMOE_CHECK_ARG(n_chunks >= 1 && n_chunks <= 64, "load_expert: n_chunks=%d outside [1, 64]", n_chunks);
  uint64_t total = 0;
  for (int c = 0; c < n_chunks; ++c) {
    ZMOE_CHECK_ARG(blocks[c] && block_sizes[c] > 0, "load_expert: empty block %d", c);
    total += original_sizes[c];
  }
  ZMOE_CHECK_ARG(total == numel, "load_expert: chunk sizes sum to %llu, expected %llu",
                 (unsigned long long)total, (unsigned long long)numel);
  zmoe::TensorStore ts;
  uint64_t pos = 0;
  for (int c = 0; c < n_chunks; ++c) {
    ts.block_off.push_back((uint32_t)pos);
    ts.block_size.push_back(block_sizes[c]);
    ts.orig_size.push_back(original_sizes[c]);
    pos += (block_sizes[c] + 15) / 16 * 16;
  }
  ts.sm_off = pos;
  ts.numel = numel;
  pos = (pos + numel + 15) / 16 * 16;
  std::vector<std::vector<uint32_t>> idx(n_chunks);
  for (int c = 0; c < n_chunks; ++c) {
    const int cap = (int)((original_sizes[c] + zmoe::kSegBytes - 1) / zmoe::kSegBytes) + 1;
    idx[c].assign(2 * (size_t)cap, 0);
    const int n = zmoe_lz4_build_index(blocks[c], block_sizes[c], original_sizes[c], zmoe::kSegBytes,
                                       idx[c].data(), cap);
    ZMOE_CHECK_ARG(n >= 1, "load_expert: block %d of expert %d tensor %d is not a valid LZ4 block (%d)", c,
                   expert, tensor, n);
    idx[c].resize(2 * (size_t)n);
    ts.idx_off.push_back(pos);
    ts.idx_n.push_back((uint32_t)n);
    pos += (idx[c].size() * 4 + 15) / 16 * 16;
  }
  ts.bytes = pos;
  std::vector<uint8_t> host(ts.bytes, 0);
  for (int c = 0; c < n_chunks; ++c) memcpy(host.data() + ts.block_off[c], blocks[c], block_sizes[c]);
  memcpy(host.data() + ts.sm_off, sm, numel);
  for (int c = 0; c < n_chunks; ++c) memcpy(host.data() + ts.idx_off[c], idx[c].data(), idx[c].size() * 4);
  if (L->host_store) {
    ZMOE_CUDA_RET(cudaHostAlloc((void**)&ts.host, ts.bytes, cudaHostAllocDefault));
    memcpy(ts.host, host.data(), ts.bytes);
  } else {
    zmoe_status st = upload((void**)&ts.dev, host.data(), ts.bytes);
    if (st != ZMOE_OK) return st;
  }
  auto& slot = L->store[expert][tensor];
  cudaFree(slot.dev);
  cudaFreeHost(slot.host);
  L->stats.store_bytes += ts.bytes - slot.bytes;
  slot = std::move(ts);
  // a re-loaded expert must be decoded again
  if (L->expert_slot[expert] >= 0) {
    L->slot_owner[L->expert_slot[expert]] = -1;
    L->expert_slot[expert] = -1;
  }
  return ZMOE_OK;
}

zmoe_status zmoe_layer_set_store(zmoe_layer* layer, int where) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "set_store: null pointer");
  ZMOE_CHECK_ARG(where == ZMOE_STORE_DEVICE || where == ZMOE_STORE_HOST, "set_store: unknown store %d", where);
  for (auto& e : L->store)
    for (auto& t : e) ZMOE_CHECK_ARG(!t.loaded(), "set_store: experts are already loaded");
  L->host_store = where == ZMOE_STORE_HOST;
  if (L->host_store && L->cfg.sm_slots > 0 && !L->sm_pool) {
    L->n_sm = L->cfg.sm_slots;
    ZMOE_CUDA_RET(cudaMalloc(&L->sm_pool, (size_t)L->n_sm * L->tensors * L->numel));
    L->sm_owner.assign(L->n_sm, -1);
    L->sm_stamp.assign(L->n_sm, 0);
  }
  return ZMOE_OK;
}

zmoe_status zmoe_layer_warm_cache(zmoe_layer* layer, const int* experts, int n, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && (n == 0 || experts), "warm_cache: null pointer");
  ZMOE_CHECK_ARG(n <= L->n_cache, "warm_cache: %d experts > %d cache slots", n, L->n_cache);
  std::vector<std::pair<int, int>> jobs;
  for (int i = 0; i < n; ++i) {
    const int e = experts[i];
    ZMOE_CHECK_ARG(e >= 0 && e < L->cfg.num_experts, "warm_cache: expert %d out of range", e);
    for (int t = 0; t < L->tensors; ++t)
      ZMOE_CHECK_ARG(L->store[e][t].loaded(), "warm_cache: expert %d not loaded", e);
    if (L->expert_slot[e] >= 0) continue;
    int slot = -1;
    for (int s2 = 0; s2 < L->n_cache; ++s2)
      if (L->slot_owner[s2] < 0) { slot = s2; break; }
    ZMOE_CHECK_ARG(slot >= 0, "warm_cache: no free cache slot");
    L->slot_owner[slot] = e;
    L->expert_slot[e] = slot;
    L->slot_admit[slot] = L->clock;
    jobs.push_back({e, slot});
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ZMOE_CUDA_RET(cudaEventRecord(L->ev_caller, s));       // free slots: nothing queued reads them, but keep order
  ZMOE_CUDA_RET(cudaStreamWaitEvent(L->ds, L->ev_caller, 0));
  zmoe_status st = L->decode_into(jobs, L->ds);
  if (st != ZMOE_OK) return st;
  ZMOE_CUDA_RET(cudaEventRecord(L->ev_decoded, L->ds));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(s, L->ev_decoded, 0));
  return L->reclaim(true);                               // the cache is warm when this returns
}

zmoe_status zmoe_layer_prefetch(zmoe_layer* layer, const int* experts, int n, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && (n == 0 || experts), "prefetch: null pointer");
  const int E = L->cfg.num_experts;
  std::vector<char> keep(E, 0);                  // experts of this call are not each other's victims
  for (int i = 0; i < n; ++i) {
    ZMOE_CHECK_ARG(experts[i] >= 0 && experts[i] < E, "prefetch: expert %d out of range", experts[i]);
    for (int t = 0; t < L->tensors; ++t)
      ZMOE_CHECK_ARG(L->store[experts[i]][t].loaded(), "prefetch: expert %d not loaded", experts[i]);
    keep[experts[i]] = 1;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  zmoe_status st = L->check_status();
  if (st != ZMOE_OK) return st;
  std::vector<std::pair<int, int>> jobs;
  for (int i = 0; i < n && L->n_cache > 0; ++i) {
    const int e = experts[i];
    if (L->expert_slot[e] >= 0) continue;
    const int slot = L->choose_victim(keep);
    if (slot < 0) break;                           // every slot holds an expert of this call
    if (L->slot_owner[slot] >= 0) { L->expert_slot[L->slot_owner[slot]] = -1; L->stats.evictions++; }
    L->slot_owner[slot] = e;
    L->expert_slot[e] = slot;
    L->slot_count[slot] = 0;
    L->slot_stamp[slot] = L->clock;
    L->slot_admit[slot] = L->clock;
    jobs.push_back({e, slot});
  }
  if (jobs.empty()) return ZMOE_OK;
  // the victims were last read by FFN work already queued on the caller's
  // stream; the decode runs after it on the decode stream, and the next FFN
  // over cache hits waits for the decode (ev_prefetch).  No host wait.
  ZMOE_CUDA_RET(cudaEventRecord(L->ev_caller, s));
  ZMOE_CUDA_RET(cudaStreamWaitEvent(L->ds, L->ev_caller, 0));
  if ((st = L->decode_into(jobs, L->ds)) != ZMOE_OK) return st;
  ZMOE_CUDA_RET(cudaEventRecord(L->ev_prefetch, L->ds));
  L->prefetch_pending = true;
  return ZMOE_OK;
}

zmoe_status zmoe_layer_forward(zmoe_layer* layer, const uint16_t* x, int T, uint16_t* out, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "forward: null layer");
  return L->forward(x, T, out, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_layer_experts(zmoe_layer* layer, const uint16_t* x_rows, const int32_t* counts_host, int rows,
                               uint16_t* y, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "experts: null layer");
  return L->experts(x_rows, counts_host, rows, y, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_layer_forward_host(zmoe_layer* layer, const uint16_t* x_host, int T, uint16_t* out_host,
                                    zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && x_host && out_host, "forward_host: null pointer");
  ZMOE_CHECK_ARG(T >= 0 && T <= L->cfg.max_tokens, "forward_host: T=%d outside [0, max_tokens]", T);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t bytes = (size_t)T * L->cfg.hidden * 2;
  if (L->submitted > 0)                                // slot 0 is shared with submit_host's steps
    for (int k = 0; k < 2; ++k) ZMOE_CUDA_RET(cudaStreamWaitEvent(s, L->out_done[k], 0));
  ZMOE_CUDA_RET(cudaMemcpyAsync(L->x_stage, x_host, bytes, cudaMemcpyHostToDevice, s));
  zmoe_status st = L->forward(L->x_stage, T, L->out_stage, s);
  if (st != ZMOE_OK) return st;
  ZMOE_CUDA_RET(cudaMemcpyAsync(out_host, L->out_stage, bytes, cudaMemcpyDeviceToHost, s));
  ZMOE_CUDA_RET(cudaStreamSynchronize(s));
  return ZMOE_OK;
}

zmoe_status zmoe_layer_submit_host(zmoe_layer* layer, const uint16_t* x_host, int T, uint16_t* out_host,
                                   zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L && x_host && out_host, "submit_host: null pointer");
  ZMOE_CHECK_ARG(T >= 0 && T <= L->cfg.max_tokens, "submit_host: T=%d outside [0, max_tokens]", T);
  return L->submit_host(x_host, T, out_host, reinterpret_cast<cudaStream_t>(stream));
}

zmoe_status zmoe_layer_join_host(zmoe_layer* layer, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "join_host: null pointer");
  if (L->submitted == 0) return ZMOE_OK;
  const int k = (int)((L->submitted - 1) & 1);         // the last step; copy_out runs its copies in order
  ZMOE_CUDA_RET(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), L->out_done[k], 0));
  return ZMOE_OK;
}

zmoe_status zmoe_layer_sync(zmoe_layer* layer, zmoe_stream_t stream) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "sync: null layer");
  ZMOE_CUDA_RET(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  zmoe_status st = L->reclaim(true);                     // decodes on the decode stream too (prefetches)
  if (st != ZMOE_OK) return st;
  if ((st = L->check_kernel_error(true)) != ZMOE_OK) return st;
  return L->fold_timing();
}

zmoe_status zmoe_layer_set_timing(zmoe_layer* layer, int enable) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "set_timing: null layer");
  L->timing = enable != 0;
  return ZMOE_OK;
}

zmoe_status zmoe_layer_reset_stats(zmoe_layer* layer) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "reset_stats: null layer");
  const uint64_t store = L->stats.store_bytes;
  L->stats = zmoe_layer_stats{};
  L->stats.store_bytes = store;
  return ZMOE_OK;
}

zmoe_status zmoe_layer_get_stats(const zmoe_layer* layer, zmoe_layer_stats* out) {
  const Layer* L = reinterpret_cast<const Layer*>(layer);
  ZMOE_CHECK_ARG(L && out, "get_stats: null pointer");
  *out = L->stats;
  return ZMOE_OK;
}

zmoe_status zmoe_layer_last_counts(const zmoe_layer* layer, int32_t* counts, int cap, int* n) {
  const Layer* L = reinterpret_cast<const Layer*>(layer);
  ZMOE_CHECK_ARG(L && n, "last_counts: null pointer");
  const int E = L->cfg.num_experts;
  *n = E;
  if (counts)
    for (int e = 0; e < E && e < cap; ++e) counts[e] = L->counts_host[e];
  return ZMOE_OK;
}

zmoe_status zmoe_layer_reset_access_counts(zmoe_layer* layer) {
  Layer* L = reinterpret_cast<Layer*>(layer);
  ZMOE_CHECK_ARG(L, "reset_access_counts: null layer");
  std::fill(L->global_count.begin(), L->global_count.end(), 0);
  std::fill(L->slot_count.begin(), L->slot_count.end(), 0);
  return ZMOE_OK;
}

zmoe_status zmoe_layer_cached_experts(const zmoe_layer* layer, int32_t* experts, int cap, int* n) {
  const Layer* L = reinterpret_cast<const Layer*>(layer);
  ZMOE_CHECK_ARG(L && n, "cached_experts: null pointer");
  int c = 0;
  for (int s = 0; s < L->n_cache; ++s)
    if (L->slot_owner[s] >= 0) {
      if (experts && c < cap) experts[c] = L->slot_owner[s];
      ++c;
    }
  *n = c;
  return ZMOE_OK;
}

}  // extern "C"
