// Expert-parallel MoE layer over NCCL, one process per GPU.
//
// Rank r owns the contiguous expert block [r*E/P, (r+1)*E/P); router, shared
// expert and tokens are data-parallel (every rank routes its own tokens).  One
// forward on every rank, all on the caller's stream except the shared expert:
//
//  1. router + permute of the local tokens: rows grouped by global expert, so
//     the rows bound for one rank are contiguous;
//  2. the shared expert on the layer's side stream (it needs only x);
//  3. per-expert counts to every rank (grouped ncclSend/ncclRecv, int32);
//  4. one host wait for the counts, which the local cache decision needs
//     anyway; the host derives the row sizes and the regroup order (rows
//     arrive as [source rank][local expert] and are regrouped by local expert);
//  5. the BF16 rows to their experts' ranks, regrouped by a row gather;
//  6. the local engine's expert stage (zmoe_layer_experts: cache decision,
//     miss decode, tcgen05 grouped FFN) -> BF16 rows;
//  7. the inverse regroup and the BF16 rows back to their tokens' ranks;
//  8. the gate-weighted combine with the shared expert.
//
// The reference runs one rank's experts through ExpertExecutor.dispatch_local
// (experts/expert_executor.py:40-84), gathering an expert's rows with a
// boolean index (csrc/dispatcher/expert_dispatcher.cpp:326-330); the exchange
// around it is the all-to-all its vendored DeepSeek expert parallelism
// implies.  NCCL is the library the process already loaded (the one
// torch.distributed uses), found with dlopen(RTLD_NOLOAD); the communicator is
// the caller's (for example ProcessGroupNCCL._comm_ptr()).  Every rank must
// call zmoe_ep_forward in the same order, as with any NCCL collective.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace zmoe {

zmoe_status launch_router(const zmoe_router_args*, cudaStream_t);
zmoe_status launch_permute(const zmoe_permute_args*, cudaStream_t);
zmoe_status launch_combine(const zmoe_combine_args*, cudaStream_t);
zmoe_status launch_gather_rows(const void*, const int32_t*, int, int, void*, cudaStream_t);

namespace {

struct Nccl {
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) return;
    n.send = reinterpret_cast<decltype(n.send)>(dlsym(h, "ncclSend"));
    n.recv = reinterpret_cast<decltype(n.recv)>(dlsym(h, "ncclRecv"));
    n.group_start = reinterpret_cast<decltype(n.group_start)>(dlsym(h, "ncclGroupStart"));
    n.group_end = reinterpret_cast<decltype(n.group_end)>(dlsym(h, "ncclGroupEnd"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.send && n.recv && n.group_start && n.group_end && n.error_string;
  });
  return n;
}

#define ZMOE_NCCL_RET(expr)                                                              \
  do {                                                                                   \
    ncclResult_t r_ = (expr);                                                            \
    if (r_ != ncclSuccess) {                                                             \
      ::zmoe::set_error("%s failed: %s", #expr, ::zmoe::nccl().error_string(r_));        \
      return ZMOE_ENCCL;                                                                 \
    }                                                                                    \
  } while (0)

template <class T>
T* dalloc(size_t n, zmoe_status* st) {
  void* p = nullptr;
  if (cudaMalloc(&p, (n ? n : 1) * sizeof(T)) != cudaSuccess) {
    set_error("cudaMalloc of %zu bytes failed", n * sizeof(T));
    *st = ZMOE_ENOMEM;
    return nullptr;
  }
  return static_cast<T*>(p);
}

template <class T>
T* halloc(size_t n, zmoe_status* st) {
  void* p = nullptr;
  if (cudaMallocHost(&p, (n ? n : 1) * sizeof(T)) != cudaSuccess) {
    set_error("cudaMallocHost of %zu bytes failed", n * sizeof(T));
    *st = ZMOE_ENOMEM;
    return nullptr;
  }
  return static_cast<T*>(p);
}

}  // namespace

struct EP {
  zmoe_layer_config cfg{};
  int rank = 0, world = 1, El = 0;
  std::vector<int> bounds;                 // expert block of rank r: [bounds[r], bounds[r + 1])
  ncclComm_t comm = nullptr;
  zmoe_layer* local = nullptr;             // this rank's experts (not owned)
  // weights
  uint16_t *w_router = nullptr, *w_sgate = nullptr, *w_shared[3] = {nullptr, nullptr, nullptr};
  float* bias = nullptr;
  // workspace (per-rank tokens T <= cfg.max_tokens, rows <= T * k, received rows <= P * T * k)
  int32_t *idx = nullptr, *counts = nullptr, *offsets = nullptr, *row_of = nullptr, *tor = nullptr;
  float *tw = nullptr, *sg = nullptr;
  uint16_t *xp = nullptr, *hsh = nullptr, *ysh = nullptr;
  int32_t* recv_counts = nullptr;          // [P * El]
  int32_t* plan_dev = nullptr;             // [2 * P * T * k]: regroup index, then its inverse
  uint16_t *recv_x = nullptr, *xg = nullptr, *yg = nullptr, *y_src = nullptr, *y_back = nullptr;
  int32_t* counts_host = nullptr;          // pinned: [E] sent counts, then [P * El] received
  int32_t* plan_host = nullptr;            // pinned regroup plan
  cudaStream_t side = nullptr;
  cudaEvent_t ev_counts = nullptr, ev_permuted = nullptr, ev_shared = nullptr, ev_plan = nullptr;
  bool plan_pending = false;
  uint64_t forwards = 0;

  ~EP() {
    for (void* p : {(void*)w_router, (void*)w_sgate, (void*)bias, (void*)w_shared[0], (void*)w_shared[1],
                    (void*)w_shared[2], (void*)idx, (void*)counts, (void*)offsets, (void*)row_of, (void*)tor,
                    (void*)tw, (void*)sg, (void*)xp, (void*)hsh, (void*)ysh, (void*)recv_counts, (void*)plan_dev,
                    (void*)recv_x, (void*)xg, (void*)yg, (void*)y_src, (void*)y_back})
      cudaFree(p);
    cudaFreeHost(counts_host);
    cudaFreeHost(plan_host);
    for (cudaEvent_t e : {ev_counts, ev_permuted, ev_shared, ev_plan})
      if (e) cudaEventDestroy(e);
    if (side) cudaStreamDestroy(side);
  }

  zmoe_status init() {
    const int E = cfg.num_experts, T = cfg.max_tokens, k = cfg.topk, H = cfg.hidden, P = world;
    bounds.resize(P + 1);
    for (int r = 0; r <= P; ++r) bounds[r] = (int)((int64_t)r * E / P);
    El = bounds[rank + 1] - bounds[rank];
    const size_t rows = (size_t)T * k, recv_rows = (size_t)P * rows;
    zmoe_status st = ZMOE_OK;
    idx = dalloc<int32_t>(rows, &st);
    tw = dalloc<float>(rows, &st);
    sg = dalloc<float>(T, &st);
    counts = dalloc<int32_t>(E, &st);
    offsets = dalloc<int32_t>(E + 1, &st);
    row_of = dalloc<int32_t>(rows, &st);
    tor = dalloc<int32_t>(rows, &st);
    xp = dalloc<uint16_t>(rows * H, &st);
    if (cfg.shared_inter > 0) {
      hsh = dalloc<uint16_t>((size_t)T * cfg.shared_inter, &st);
      ysh = dalloc<uint16_t>((size_t)T * H, &st);
    }
    recv_counts = dalloc<int32_t>((size_t)P * El, &st);
    plan_dev = dalloc<int32_t>(2 * recv_rows, &st);
    recv_x = dalloc<uint16_t>(recv_rows * H, &st);
    xg = dalloc<uint16_t>(recv_rows * H, &st);
    yg = dalloc<uint16_t>(recv_rows * H, &st);
    y_src = dalloc<uint16_t>(recv_rows * H, &st);
    y_back = dalloc<uint16_t>(rows * H, &st);
    counts_host = halloc<int32_t>((size_t)E + (size_t)P * El, &st);
    plan_host = halloc<int32_t>(2 * recv_rows, &st);
    if (st != ZMOE_OK) return st;
    ZMOE_CUDA_RET(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&ev_counts, &ev_permuted, &ev_shared, &ev_plan})
      ZMOE_CUDA_RET(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    return ZMOE_OK;
  }

  zmoe_status forward(const uint16_t* x, int T, uint16_t* out, cudaStream_t s);
  // One all-to-all of `elems` bytes-per-item blocks: block r of `send` (items
  // [soff[r], soff[r] + scnt[r])) goes to rank r, block r of `recv` comes
  // from it.  A single rank copies on the stream.
  zmoe_status exchange(const void* send, const int* soff, const int* scnt, void* recv, const int* roff,
                       const int* rcnt, size_t item_elems, ncclDataType_t type, size_t elem_bytes, cudaStream_t s);
};

zmoe_status EP::exchange(const void* send, const int* soff, const int* scnt, void* recv, const int* roff,
                         const int* rcnt, size_t item_elems, ncclDataType_t type, size_t elem_bytes, cudaStream_t s) {
  const size_t ib = item_elems * elem_bytes;
  if (world == 1) {
    if (scnt[0] > 0)
      ZMOE_CUDA_RET(cudaMemcpyAsync(static_cast<char*>(recv) + roff[0] * ib,
                                    static_cast<const char*>(send) + soff[0] * ib, scnt[0] * ib,
                                    cudaMemcpyDeviceToDevice, s));
    return ZMOE_OK;
  }
  const Nccl& N = nccl();
  ZMOE_NCCL_RET(N.group_start());
  for (int r = 0; r < world; ++r) {
    ZMOE_NCCL_RET(N.send(static_cast<const char*>(send) + soff[r] * ib, (size_t)scnt[r] * item_elems, type, r, comm,
                         s));
    ZMOE_NCCL_RET(N.recv(static_cast<char*>(recv) + roff[r] * ib, (size_t)rcnt[r] * item_elems, type, r, comm, s));
  }
  ZMOE_NCCL_RET(N.group_end());
  return ZMOE_OK;
}

zmoe_status EP::forward(const uint16_t* x, int T, uint16_t* out, cudaStream_t s) {
  const int E = cfg.num_experts, k = cfg.topk, H = cfg.hidden, P = world;
  ZMOE_CHECK_ARG(x && out, "ep_forward: null pointer");
  ZMOE_CHECK_ARG(T >= 0 && T <= cfg.max_tokens, "ep_forward: T=%d outside [0, max_tokens=%d]", T, cfg.max_tokens);
  ZMOE_CHECK_ARG(w_router, "ep_forward: router weights not set");
  zmoe_status st;
  // 1. router + permute over the global experts (T may be 0 on a rank: it
  //    still takes part in every exchange)
  if (T > 0) {
    zmoe_router_args ra{};
    ra.x = x; ra.w = w_router; ra.bias = bias; ra.w_shared_gate = w_sgate;
    ra.T = T; ra.H = H; ra.E = E; ra.k = k; ra.mode = cfg.route_mode;
    ra.norm_topk_prob = cfg.norm_topk_prob; ra.scaling = cfg.scaling;
    ra.logits = nullptr; ra.topk_idx = idx; ra.topk_w = tw; ra.shared_gate = w_sgate ? sg : nullptr;
    if ((st = launch_router(&ra, s)) != ZMOE_OK) return st;
    zmoe_permute_args pa{};
    pa.topk_idx = idx; pa.x = x; pa.T = T; pa.H = H; pa.E = E; pa.k = k;
    pa.capacity = cfg.route_mode == ZMOE_ROUTE_SWITCH ? cfg.capacity : 0;
    pa.seq_len = cfg.seq_len > 0 ? cfg.seq_len : T;
    pa.counts = counts; pa.offsets = offsets; pa.row_of = row_of; pa.token_of_row = tor; pa.xp = xp;
    if ((st = launch_permute(&pa, s)) != ZMOE_OK) return st;
  } else {
    ZMOE_CUDA_RET(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, s));
  }
  // 2. the shared expert beside the exchange
  const bool shared = T > 0 && cfg.shared_inter > 0 && w_shared[0];
  if (shared) {
    ZMOE_CUDA_RET(cudaEventRecord(ev_permuted, s));
    ZMOE_CUDA_RET(cudaStreamWaitEvent(side, ev_permuted, 0));
    zmoe_ffn_args fa{};
    const uint16_t* tab[3] = {w_shared[0], w_shared[1], w_shared[2]};
    fa.x = x; fa.w = tab; fa.offsets = nullptr; fa.G = 1; fa.rows_total = T; fa.H = H;
    fa.I = cfg.shared_inter; fa.kind = 0; fa.h = hsh; fa.y = ysh;
    if ((st = launch_expert_ffn(&fa, side)) != ZMOE_OK) return st;
    ZMOE_CUDA_RET(cudaEventRecord(ev_shared, side));
  }
  // 3. counts: the block of rank r's experts goes to r
  {
    std::vector<int> sc(P), rc(P, El), ro(P);
    for (int r = 0; r < P; ++r) {
      sc[r] = bounds[r + 1] - bounds[r];
      ro[r] = r * El;
    }
    if ((st = exchange(counts, bounds.data(), sc.data(), recv_counts, ro.data(), rc.data(), 1, ncclInt32, 4, s)) !=
        ZMOE_OK)
      return st;
  }
  // 4. the host learns the counts (its pinned plan buffer is free once the
  //    previous forward's plan copy has run)
  if (plan_pending) {
    ZMOE_CUDA_RET(cudaEventSynchronize(ev_plan));
    plan_pending = false;
  }
  ZMOE_CUDA_RET(cudaMemcpyAsync(counts_host, counts, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, s));
  ZMOE_CUDA_RET(cudaMemcpyAsync(counts_host + E, recv_counts, sizeof(int32_t) * P * El, cudaMemcpyDeviceToHost, s));
  ZMOE_CUDA_RET(cudaEventRecord(ev_counts, s));
  ZMOE_CUDA_RET(cudaEventSynchronize(ev_counts));
  const int32_t* c_send = counts_host;
  const int32_t* c_recv = counts_host + E;            // [P][El]
  std::vector<int> send_rows(P, 0), recv_rows(P, 0), send_off(P + 1, 0), recv_off(P + 1, 0);
  std::vector<int32_t> counts_local(El, 0);
  for (int r = 0; r < P; ++r) {
    for (int e = bounds[r]; e < bounds[r + 1]; ++e) send_rows[r] += c_send[e];
    for (int e = 0; e < El; ++e) {
      recv_rows[r] += c_recv[(size_t)r * El + e];
      counts_local[e] += c_recv[(size_t)r * El + e];
    }
    send_off[r + 1] = send_off[r] + send_rows[r];
    recv_off[r + 1] = recv_off[r] + recv_rows[r];
  }
  const int n_send = send_off[P], n_recv = recv_off[P];
  ZMOE_CHECK_ARG(n_recv <= P * cfg.max_tokens * k, "ep_forward: %d rows received, more than P*max_tokens*topk",
                 n_recv);
  // regroup: received [source rank][local expert] -> [local expert][source rank]
  int32_t* index = plan_host;
  int32_t* inverse = plan_host + n_recv;
  {
    int i = 0;
    for (int e = 0; e < El; ++e)
      for (int r = 0; r < P; ++r) {
        int start = recv_off[r];
        for (int e2 = 0; e2 < e; ++e2) start += c_recv[(size_t)r * El + e2];
        for (int j = 0; j < c_recv[(size_t)r * El + e]; ++j) index[i++] = start + j;
      }
    for (int g = 0; g < n_recv; ++g) inverse[index[g]] = g;
  }
  if (n_recv > 0) {
    ZMOE_CUDA_RET(cudaMemcpyAsync(plan_dev, plan_host, sizeof(int32_t) * 2 * (size_t)n_recv,
                                  cudaMemcpyHostToDevice, s));
    ZMOE_CUDA_RET(cudaEventRecord(ev_plan, s));
    plan_pending = true;
  }
  // 5. rows out, regrouped by local expert
  if ((st = exchange(xp, send_off.data(), send_rows.data(), recv_x, recv_off.data(), recv_rows.data(), (size_t)H,
                     ncclBfloat16, 2, s)) != ZMOE_OK)
    return st;
  if (n_recv > 0) {
    if ((st = launch_gather_rows(recv_x, plan_dev, n_recv, H * 2, xg, s)) != ZMOE_OK) return st;
  }
  // 6. this rank's experts (always called, so the engine's bookkeeping sees every step)
  if ((st = zmoe_layer_experts(local, xg, counts_local.data(), n_recv, yg, s)) != ZMOE_OK) return st;
  // 7. rows back in the order they left
  if (n_recv > 0) {
    if ((st = launch_gather_rows(yg, plan_dev + n_recv, n_recv, H * 2, y_src, s)) != ZMOE_OK) return st;
  }
  if ((st = exchange(y_src, recv_off.data(), recv_rows.data(), y_back, send_off.data(), send_rows.data(), (size_t)H,
                     ncclBfloat16, 2, s)) != ZMOE_OK)
    return st;
  // 8. combine on the local tokens
  if (shared) ZMOE_CUDA_RET(cudaStreamWaitEvent(s, ev_shared, 0));
  if (T > 0) {
    zmoe_combine_args ca{};
    ca.y = y_back; ca.y_shared = shared ? ysh : nullptr;
    ca.shared_gate = (shared && w_sgate) ? sg : nullptr; ca.row_of = row_of; ca.topk_w = tw; ca.x = x;
    ca.T = T; ca.H = H; ca.k = k; ca.mode = cfg.route_mode; ca.out = out;
    if ((st = launch_combine(&ca, s)) != ZMOE_OK) return st;
  }
  (void)n_send;
  ++forwards;
  return ZMOE_OK;
}

}  // namespace zmoe

using zmoe::EP;

extern "C" {

zmoe_status zmoe_ep_create(const zmoe_ep_config* cfg, zmoe_layer* local, zmoe_ep** out) {
  ZMOE_CHECK_ARG(cfg && local && out, "ep_create: null pointer");
  *out = nullptr;
  ZMOE_CHECK_ARG(cfg->world >= 1 && cfg->rank >= 0 && cfg->rank < cfg->world, "ep_create: rank %d of %d",
                 cfg->rank, cfg->world);
  ZMOE_CHECK_ARG(cfg->nccl_comm || cfg->world == 1, "ep_create: no NCCL communicator");
  const zmoe_layer_config& c = cfg->layer;
  ZMOE_CHECK_ARG(c.hidden > 0 && c.hidden % 256 == 0, "ep_create: hidden=%d must be a positive multiple of 256",
                 c.hidden);
  ZMOE_CHECK_ARG(c.num_experts >= cfg->world && c.num_experts <= 256, "ep_create: %d experts over %d ranks",
                 c.num_experts, cfg->world);
  ZMOE_CHECK_ARG(c.topk >= 1 && c.topk <= 8 && c.topk <= c.num_experts, "ep_create: bad topk=%d", c.topk);
  ZMOE_CHECK_ARG(c.max_tokens >= 1, "ep_create: max_tokens must be >= 1");
  ZMOE_CHECK_ARG(c.route_mode >= 0 && c.route_mode <= 2, "ep_create: bad route_mode");
  ZMOE_CHECK_ARG(c.shared_inter == 0 || c.shared_inter % 8 == 0, "ep_create: shared_inter must be a multiple of 8");
  if (cfg->world > 1 && !zmoe::nccl().ok) {
    zmoe::set_error("ep_create: NCCL is not loaded in this process (libnccl.so.2, the library of the "
                    "communicator's owner)");
    return ZMOE_ENCCL;
  }
  auto* ep = new EP();
  ep->cfg = c;
  ep->rank = cfg->rank;
  ep->world = cfg->world;
  ep->comm = reinterpret_cast<ncclComm_t>(cfg->nccl_comm);
  ep->local = local;
  zmoe_status st = ep->init();
  if (st != ZMOE_OK) {
    delete ep;
    return st;
  }
  *out = reinterpret_cast<zmoe_ep*>(ep);
  return ZMOE_OK;
}

zmoe_status zmoe_ep_destroy(zmoe_ep* ep) {
  delete reinterpret_cast<EP*>(ep);
  return ZMOE_OK;
}

static zmoe_status ep_upload(void** dst, const void* src, size_t bytes) {
  cudaFree(*dst);
  *dst = nullptr;
  ZMOE_CUDA_RET(cudaMalloc(dst, bytes));
  ZMOE_CUDA_RET(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
  return ZMOE_OK;
}

zmoe_status zmoe_ep_set_router(zmoe_ep* ep, const uint16_t* w_router, const float* bias,
                               const uint16_t* w_shared_gate) {
  EP* P = reinterpret_cast<EP*>(ep);
  ZMOE_CHECK_ARG(P && w_router, "ep_set_router: null pointer");
  const size_t H = P->cfg.hidden, E = P->cfg.num_experts;
  zmoe_status st = ep_upload((void**)&P->w_router, w_router, E * H * 2);
  if (st == ZMOE_OK && bias) st = ep_upload((void**)&P->bias, bias, E * 4);
  if (st == ZMOE_OK && w_shared_gate) st = ep_upload((void**)&P->w_sgate, w_shared_gate, H * 2);
  return st;
}

zmoe_status zmoe_ep_set_shared(zmoe_ep* ep, const uint16_t* gate, const uint16_t* up, const uint16_t* down) {
  EP* P = reinterpret_cast<EP*>(ep);
  ZMOE_CHECK_ARG(P && gate && up && down, "ep_set_shared: null pointer");
  ZMOE_CHECK_ARG(P->cfg.shared_inter > 0, "ep_set_shared: layer has no shared expert");
  const size_t n = (size_t)P->cfg.hidden * P->cfg.shared_inter * 2;
  const uint16_t* src[3] = {gate, up, down};
  for (int i = 0; i < 3; ++i) {
    zmoe_status st = ep_upload((void**)&P->w_shared[i], src[i], n);
    if (st != ZMOE_OK) return st;
  }
  return ZMOE_OK;
}

zmoe_status zmoe_ep_forward(zmoe_ep* ep, const uint16_t* x, int T, uint16_t* out, zmoe_stream_t stream) {
  EP* P = reinterpret_cast<EP*>(ep);
  ZMOE_CHECK_ARG(P, "ep_forward: null handle");
  return P->forward(x, T, out, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
