// Python module `ZipMoE`: the reference's operator surface for the expert path
// (csrc/binding/bindings.cpp:17-222) with the same two classes, method names,
// argument names and order, over the C ABI of libzmoe.so.
//
//  * zipmoe_prefetch_handle keeps the reference's on-disk offload format: the
//    `zipmoe_param` file (every append padded to 4096 bytes,
//    TensorEngine::write_compressed_append, csrc/tensor_engine/tensor_engine.cpp:139-165)
//    and the `zipmoe_index` binary index (ZipMoETensorIndex::Serialize /
//    Deserialize and the TensorStorageMeta stream operators,
//    csrc/base/zipmoe_tensor_index.cpp:22-184).  Files written by either
//    implementation are read by the other.
//  * expert_dispatcher runs enqueued experts on the GPU: one layer engine per MoE
//    layer keeps the layer's experts compressed in HBM, keeps decoded experts in
//    a cache, decodes misses with the fused decoder and runs the tcgen05 grouped
//    FFN (ExpertDispatcher, csrc/dispatcher/expert_dispatcher.cpp:149-515).
//
// Differences that callers can see: errors raise RuntimeError instead of
// aborting the process; there are no worker threads (num_compute_threads only
// sizes the offline compression pool, bind_core is accepted and ignored);
// ZSTD is not supported; wait_expert returns results in enqueue order.
#include <torch/extension.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <future>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "zmoe.h"

namespace py = pybind11;

namespace zipmoe {

[[noreturn]] void fail(const std::string& what) { throw std::runtime_error("[ZipMoE] " + what); }

void check(zmoe_status st, const char* what) {
  if (st != ZMOE_OK) fail(std::string(what) + ": " + zmoe_last_error());
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}

constexpr uint64_t kPage = 4096;                    // OS_PAGE_SIZE of the reference
constexpr const char* kIndexName = "zipmoe_index";  // ZIPMOE_INDEX_NAME

// ---------------------------------------------------------------------------
// zipmoe_index
// ---------------------------------------------------------------------------
struct Meta {
  uint32_t id = 0;
  std::vector<int64_t> shape;
  uint64_t size = 0, num_elements = 0;
  uint8_t pinned = 0, requires_grad = 0;
  int8_t dtype = 0, device_index = -1, device_type = 0, layout = 0;
  uint32_t offload_file_id = 0;
  int32_t num_file_chunks = 0;
  std::vector<uint64_t> exp_file_offsets, compressed_sizes, original_sizes;
  uint64_t sm_file_offset = 0, sm_size = 0;
  bool sparse() const { return sm_size > 0; }     // dense tensors keep sm_size = 0
};

struct Writer {
  std::string buf;
  template <class T>
  void put(T v) { buf.append(reinterpret_cast<const char*>(&v), sizeof(T)); }
};

struct Reader {
  const std::string& buf;
  size_t pos = 0;
  template <class T>
  T get() {
    if (pos + sizeof(T) > buf.size()) fail("zipmoe_index is truncated");
    T v;
    std::memcpy(&v, buf.data() + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
};

void put_meta(Writer& w, const Meta& m) {
  w.put<uint32_t>(m.id);
  w.put<int64_t>((int64_t)m.shape.size());
  for (int64_t d : m.shape) w.put<int64_t>(d);
  w.put<uint64_t>(m.size);
  w.put<uint64_t>(m.num_elements);
  w.put<uint8_t>(m.pinned);
  w.put<uint8_t>(m.requires_grad);
  w.put<int8_t>(m.dtype);
  w.put<int8_t>(m.device_index);
  w.put<int8_t>(m.device_type);
  w.put<int8_t>(m.layout);
  w.put<uint32_t>(m.offload_file_id);
  w.put<int32_t>(m.num_file_chunks);
  for (const auto* a : {&m.exp_file_offsets, &m.compressed_sizes, &m.original_sizes}) {
    w.put<uint32_t>((uint32_t)a->size());
    for (uint64_t v : *a) w.put<uint64_t>(v);
  }
  w.put<uint64_t>(m.sm_file_offset);
  w.put<uint64_t>(m.sm_size);
}

Meta get_meta(Reader& r) {
  Meta m;
  m.id = r.get<uint32_t>();
  const int64_t nd = r.get<int64_t>();
  if (nd < 0 || nd > 64) fail("zipmoe_index: bad ndim");
  for (int64_t i = 0; i < nd; ++i) m.shape.push_back(r.get<int64_t>());
  m.size = r.get<uint64_t>();
  m.num_elements = r.get<uint64_t>();
  m.pinned = r.get<uint8_t>();
  m.requires_grad = r.get<uint8_t>();
  m.dtype = r.get<int8_t>();
  m.device_index = r.get<int8_t>();
  m.device_type = r.get<int8_t>();
  m.layout = r.get<int8_t>();
  m.offload_file_id = r.get<uint32_t>();
  m.num_file_chunks = r.get<int32_t>();
  for (auto* a : {&m.exp_file_offsets, &m.compressed_sizes, &m.original_sizes}) {
    const uint32_t k = r.get<uint32_t>();
    if (k > (1u << 20)) fail("zipmoe_index: bad array length");
    for (uint32_t i = 0; i < k; ++i) a->push_back(r.get<uint64_t>());
  }
  m.sm_file_offset = r.get<uint64_t>();
  m.sm_size = r.get<uint64_t>();
  return m;
}

struct Index {
  std::vector<uint32_t> order;                   // insertion order (the writer's entry order)
  std::unordered_map<uint32_t, Meta> map;

  bool has(uint32_t k) const { return map.count(k) != 0; }
  const Meta& at(uint32_t k) const {
    auto it = map.find(k);
    if (it == map.end()) fail("tensor " + std::to_string(k) + " is not in the index");
    return it->second;
  }
  void insert(uint32_t k, Meta m) {
    if (!map.count(k)) order.push_back(k);
    map[k] = std::move(m);
  }
  std::string serialize() const {
    Writer w;
    w.put<uint32_t>((uint32_t)order.size());
    for (uint32_t k : order) {
      w.put<uint32_t>(k);
      put_meta(w, map.at(k));
    }
    return w.buf;
  }
  void deserialize(const std::string& data) {
    order.clear();
    map.clear();
    Reader r{data};
    const uint32_t n = r.get<uint32_t>();
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t k = r.get<uint32_t>();
      insert(k, get_meta(r));
    }
  }
};

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail("cannot open " + path);
  return std::string(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

void write_file(const std::string& path, const std::string& data) {
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  if (!f) fail("cannot write " + path);
  f.write(data.data(), (std::streamsize)data.size());
  if (!f) fail("write failed: " + path);
}

// ---------------------------------------------------------------------------
// zipmoe_param
// ---------------------------------------------------------------------------
struct ParamFile {
  std::string path;
  int fd = -1;

  ~ParamFile() {
    if (fd >= 0) ::close(fd);
  }
  // Appends data and zero padding to the next 4096-byte boundary; returns the
  // offset the data starts at.
  uint64_t append(const void* data, size_t n) {
    FILE* f = std::fopen(path.c_str(), "ab");
    if (!f) fail("cannot open " + path + " for appending");
    std::fseek(f, 0, SEEK_END);
    const long start = std::ftell(f);
    bool ok = start >= 0 && std::fwrite(data, 1, n, f) == n;
    const uint64_t end = (uint64_t)start + n;
    const uint64_t pad = (kPage - end % kPage) % kPage;
    static const char zeros[kPage] = {};
    ok = ok && std::fwrite(zeros, 1, pad, f) == pad;
    ok = (std::fclose(f) == 0) && ok;
    if (!ok) fail("append to " + path + " failed");
    return (uint64_t)start;
  }
  void open_read() {
    if (fd >= 0) return;
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) fail("cannot open " + path);
  }
  void read(uint64_t off, void* dst, size_t n) const {
    if (fd < 0) fail("offload file is not open (call open_offload_file)");
    size_t done = 0;
    while (done < n) {
      const ssize_t r = ::pread(fd, static_cast<char*>(dst) + done, n - done, (off_t)(off + done));
      if (r <= 0) fail("read of " + path + " failed");
      done += (size_t)r;
    }
  }
};

// ---------------------------------------------------------------------------
// state shared by the handle and the dispatchers (the reference keeps it in
// process-wide singletons too: kTensorIndex, kZipMoETensorEngine, ...)
// ---------------------------------------------------------------------------
struct Config {
  std::string code_type = "LZ4HC", caching_algorithm = "ZipMoE";
  double device_memory_ratio = 0.5, gpu_pool_ratio = 1.0, state_margin = 0.1;
  int num_compute_threads = 1, num_file_chunks = 3, prefetcher_topk = 0, expert_topk = 1;
  size_t num_elements_per_expert = 0, num_tensors_per_expert = 3;
  int num_expert_layers = 1, num_experts = 1;
  int lz4_accel = 1, lz4hc_level = 9;
  bool gpu_encode = false;   // batch_offload encodes LZ4HC chunks on the GPU (zmoe_lz4_encode_chunks)
  int gpu_encode_attempts = 256;
};

struct Store {
  std::mutex mu;
  Config cfg;
  std::string prefix;
  Index index;
  bool index_loaded = false;
  ParamFile file;
  std::unordered_map<uint32_t, torch::Tensor> tensors;   // registered parameters
  std::unordered_map<uintptr_t, uint32_t> ptr_to_id;
  std::vector<std::tuple<std::string, std::vector<std::vector<uint32_t>>>> topology;
  std::vector<std::function<void()>> on_reset_counts;
  uint64_t generation = 0;
};

std::shared_ptr<Store> g_store;                    // the live handle's store

std::shared_ptr<Store> store_or_fail() {
  if (!g_store) fail("no zipmoe_prefetch_handle: create one before the expert_dispatcher");
  return g_store;
}

cudaStream_t current_stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

std::vector<uint8_t> read_bytes(const Store& s, uint64_t off, size_t n) {
  std::vector<uint8_t> v(n);
  if (n) s.file.read(off, v.data(), n);
  return v;
}

// Host copies of a sparse tensor's LZ4 blocks and sign+mantissa plane.
struct HostPlanes {
  std::vector<std::vector<uint8_t>> blocks;
  std::vector<uint32_t> block_sizes, original_sizes;
  std::vector<uint8_t> sm;
};

HostPlanes read_planes(const Store& s, const Meta& m) {
  if (!m.sparse()) fail("tensor " + std::to_string(m.id) + " is dense");
  const int n = m.num_file_chunks;
  if (n <= 0 || (int)m.compressed_sizes.size() != n || (int)m.original_sizes.size() != n ||
      (int)m.exp_file_offsets.size() != n)
    fail("tensor " + std::to_string(m.id) + ": inconsistent chunk arrays");
  HostPlanes p;
  uint64_t total = 0;
  for (int c = 0; c < n; ++c) {
    if (m.compressed_sizes[c] > 0xffffffffull || m.original_sizes[c] > 0x3fffffffull) fail("chunk too large");
    p.blocks.push_back(read_bytes(s, m.exp_file_offsets[c], m.compressed_sizes[c]));
    p.block_sizes.push_back((uint32_t)m.compressed_sizes[c]);
    p.original_sizes.push_back((uint32_t)m.original_sizes[c]);
    total += m.original_sizes[c];
  }
  if (total != m.num_elements || m.sm_size != m.num_elements)
    fail("tensor " + std::to_string(m.id) + ": chunk sizes do not add up to num_elements");
  p.sm = read_bytes(s, m.sm_file_offset, m.sm_size);
  return p;
}

torch::ScalarType scalar_type_of(const Meta& m) { return static_cast<torch::ScalarType>(m.dtype); }

// Decode one sparse tensor on the current GPU into a new BF16 tensor.
torch::Tensor decode_tensor(const Store& s, const Meta& m) {
  HostPlanes p = read_planes(s, m);
  const int n = (int)p.blocks.size();
  const auto dev = torch::Device(torch::kCUDA, c10::cuda::current_device());
  auto u8 = torch::TensorOptions().dtype(torch::kUInt8);
  auto i32 = torch::TensorOptions().dtype(torch::kInt32);
  // blocks (16-byte aligned), sign+mantissa, slice indexes, map scratch, descriptors, status
  std::vector<uint64_t> boff(n), ioff(n);
  std::vector<std::vector<uint32_t>> idx(n);
  uint64_t pos = 0;
  for (int c = 0; c < n; ++c) {
    boff[c] = pos;
    pos += (p.block_sizes[c] + 15) / 16 * 16;
    const int cap = (int)((p.original_sizes[c] + ZMOE_SLICE_BYTES - 1) / ZMOE_SLICE_BYTES) + 1;
    idx[c].resize(2 * (size_t)cap);
    const int k = zmoe_lz4_build_index(p.blocks[c].data(), p.block_sizes[c], p.original_sizes[c], ZMOE_SLICE_BYTES,
                                       idx[c].data(), cap);
    if (k < 0) fail("tensor " + std::to_string(m.id) + ": malformed LZ4 block (index walk " + std::to_string(k) + ")");
    idx[c].resize(2 * (size_t)k);
  }
  auto hb = torch::zeros({(int64_t)std::max<uint64_t>(pos, 16)}, u8);
  for (int c = 0; c < n; ++c) std::memcpy(hb.data_ptr<uint8_t>() + boff[c], p.blocks[c].data(), p.block_sizes[c]);
  uint64_t ipos = 0;
  for (int c = 0; c < n; ++c) { ioff[c] = ipos; ipos += idx[c].size(); }
  auto hi = torch::empty({(int64_t)std::max<uint64_t>(ipos, 2)}, i32);
  for (int c = 0; c < n; ++c)
    std::memcpy(hi.data_ptr<int32_t>() + ioff[c], idx[c].data(), idx[c].size() * 4);
  auto db = hb.to(dev);
  auto dsm = torch::from_blob(p.sm.data(), {(int64_t)p.sm.size()}, u8).to(dev);
  auto di = hi.to(dev);
  std::vector<uint64_t> moff(n);
  uint64_t mbytes = 0;
  for (int c = 0; c < n; ++c) { moff[c] = mbytes; mbytes += zmoe_decode_scratch_bytes(p.original_sizes[c]); }
  auto map = torch::empty({(int64_t)(mbytes / 4)}, i32.device(dev));
  auto out = torch::empty({(int64_t)m.num_elements}, torch::TensorOptions().dtype(torch::kBFloat16).device(dev));
  std::vector<zmoe_chunk> d(n);
  uint64_t e0 = 0;
  for (int c = 0; c < n; ++c) {
    d[c].src = db.data_ptr<uint8_t>() + boff[c];
    d[c].sm = dsm.data_ptr<uint8_t>() + e0;
    d[c].dst = reinterpret_cast<uint16_t*>(out.data_ptr()) + e0;
    d[c].index = reinterpret_cast<const uint32_t*>(di.data_ptr<int32_t>() + ioff[c]);
    d[c].map = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(map.data_ptr<int32_t>()) + moff[c]);
    d[c].src_size = p.block_sizes[c];
    d[c].out_size = p.original_sizes[c];
    d[c].n_index = (uint32_t)(idx[c].size() / 2);
    d[c].seg_bytes = ZMOE_SLICE_BYTES;
    e0 += p.original_sizes[c];
  }
  auto hd = torch::from_blob(d.data(), {(int64_t)(n * sizeof(zmoe_chunk))}, u8).to(dev);
  auto st = torch::full({n}, -1, i32.device(dev));
  check(zmoe_decode_chunks(reinterpret_cast<const zmoe_chunk*>(hd.data_ptr<uint8_t>()), n, st.data_ptr<int32_t>(),
                           current_stream()),
        "zmoe_decode_chunks");
  auto sh = st.cpu();                               // waits for the decode
  for (int c = 0; c < n; ++c)
    if (sh.data_ptr<int32_t>()[c] != 0)
      fail("tensor " + std::to_string(m.id) + ": chunk " + std::to_string(c) + " failed to decode (status " +
           std::to_string(sh.data_ptr<int32_t>()[c]) + ")");
  std::vector<int64_t> shape(m.shape.begin(), m.shape.end());
  return out.view(shape);
}

torch::Tensor read_dense(const Store& s, const Meta& m) {
  std::vector<uint8_t> raw = read_bytes(s, m.sm_file_offset, m.size);
  const auto t = scalar_type_of(m);
  std::vector<int64_t> shape(m.shape.begin(), m.shape.end());
  auto host = torch::from_blob(raw.data(), shape, torch::TensorOptions().dtype(t)).clone();
  return host.to(torch::Device(torch::kCUDA, c10::cuda::current_device()));
}

int compress_codec(const std::string& code) {
  if (code == "LZ4") return ZMOE_CODEC_LZ4;
  if (code == "LZ4HC") return ZMOE_CODEC_LZ4HC;
  fail("CODE_TYPE '" + code + "' is not supported (LZ4 and LZ4HC are)");
}

std::vector<uint8_t> compress_chunk(const Config& cfg, const uint8_t* src, size_t n) {
  if (n > 0x7fffffff) fail("exponent chunk too large");
  const int codec = compress_codec(cfg.code_type);
  const int level = codec == ZMOE_CODEC_LZ4 ? cfg.lz4_accel : cfg.lz4hc_level;
  const int bound = zmoe_lz4_compress_bound((int)n);
  std::vector<uint8_t> out((size_t)std::max(bound, 16));
  const int got = zmoe_lz4_compress(src, (int)n, out.data(), (int)out.size(), codec, level);
  if (got <= 0) fail("LZ4 compression failed");
  out.resize((size_t)got);
  return out;
}

// LZ4 blocks of host chunks, encoded on the current GPU: every chunk of a
// group of up to 512 MiB goes in one zmoe_lz4_encode_chunks call (replaces
// the compute pool's per-chunk LZ4HCcompressor::compress,
// csrc/tensor_engine/tensor_engine.cpp:105-136).
std::vector<std::vector<uint8_t>> gpu_compress_chunks(const std::vector<std::pair<const uint8_t*, size_t>>& chunks,
                                                      int attempts) {
  std::vector<std::vector<uint8_t>> out(chunks.size());
  const int dev = c10::cuda::current_device();
  const auto u8 = torch::TensorOptions().dtype(torch::kUInt8);
  const auto on_dev = u8.device(torch::kCUDA, dev);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  const uint64_t kGroupBytes = 512ull << 20;
  size_t g0 = 0;
  while (g0 < chunks.size()) {
    size_t g1 = g0;
    uint64_t in_total = 0, cap_total = 0, scr_total = 0;
    std::vector<uint64_t> in_off, cap_off, scr_off, cap;
    while (g1 < chunks.size() && g1 - g0 < 65535 && (g1 == g0 || in_total + chunks[g1].second <= kGroupBytes)) {
      const uint64_t n = chunks[g1].second;
      if (n > (1u << 30)) fail("exponent chunk too large for the GPU encoder (1 GiB at most)");
      in_off.push_back(in_total);
      cap_off.push_back(cap_total);
      scr_off.push_back(scr_total);
      cap.push_back(n + n / 255 + 16);
      in_total += (n + 15) / 16 * 16;
      cap_total += cap.back();
      scr_total += (zmoe_lz4_encode_scratch_bytes((uint32_t)n) + 15) / 16 * 16;
      ++g1;
    }
    const size_t k = g1 - g0;
    torch::Tensor hin = torch::empty({(int64_t)std::max<uint64_t>(in_total, 16)}, u8.pinned_memory(true));
    for (size_t c = 0; c < k; ++c)
      if (chunks[g0 + c].second) std::memcpy(hin.data_ptr<uint8_t>() + in_off[c], chunks[g0 + c].first, chunks[g0 + c].second);
    torch::Tensor din = hin.to(on_dev, /*non_blocking=*/true);
    torch::Tensor dout = torch::empty({(int64_t)cap_total}, on_dev);
    torch::Tensor dscr = torch::empty({(int64_t)std::max<uint64_t>(scr_total, 16)}, on_dev);
    std::vector<zmoe_enc_chunk> desc(k);
    for (size_t c = 0; c < k; ++c) {
      desc[c].src = din.data_ptr<uint8_t>() + in_off[c];
      desc[c].dst = dout.data_ptr<uint8_t>() + cap_off[c];
      desc[c].scratch = dscr.data_ptr<uint8_t>() + scr_off[c];
      desc[c].src_size = (uint32_t)chunks[g0 + c].second;
      desc[c].dst_capacity = (uint32_t)cap[c];
    }
    torch::Tensor hdesc = torch::from_blob(desc.data(), {(int64_t)(k * sizeof(zmoe_enc_chunk))}, u8);
    torch::Tensor ddesc = hdesc.to(on_dev);
    torch::Tensor dsizes = torch::zeros({(int64_t)k}, on_dev.dtype(torch::kInt32));
    check(zmoe_lz4_encode_chunks(reinterpret_cast<const zmoe_enc_chunk*>(ddesc.data_ptr()), (int)k, attempts,
                                 reinterpret_cast<uint32_t*>(dsizes.data_ptr<int32_t>()),
                                 reinterpret_cast<zmoe_stream_t>(stream)),
          "zmoe_lz4_encode_chunks");
    torch::Tensor hsizes = dsizes.cpu();
    torch::Tensor hout = dout.cpu();
    for (size_t c = 0; c < k; ++c) {
      const int32_t got = hsizes.data_ptr<int32_t>()[c];
      if (got <= 0) fail("GPU LZ4 encoding failed");
      const uint8_t* b = hout.data_ptr<uint8_t>() + cap_off[c];
      out[g0 + c].assign(b, b + got);
    }
    g0 = g1;
  }
  return out;
}

// ---------------------------------------------------------------------------
// zipmoe_prefetch_handle
// ---------------------------------------------------------------------------
struct ChunkArrays {
  std::vector<std::pair<const uint8_t*, size_t>> chunks;
  const uint8_t* sm = nullptr;
  size_t sm_size = 0;
};

ChunkArrays view_arrays(const std::vector<py::array_t<uint8_t, py::array::c_style | py::array::forcecast>>& exp,
                        const py::array_t<uint8_t, py::array::c_style | py::array::forcecast>& sm) {
  ChunkArrays a;
  for (const auto& c : exp) a.chunks.push_back({c.data(), (size_t)c.size()});
  a.sm = sm.data();
  a.sm_size = (size_t)sm.size();
  return a;
}

Meta meta_of(uint32_t id, const torch::Tensor& t, int num_file_chunks) {
  Meta m;
  m.id = id;
  m.shape = t.sizes().vec();
  m.size = t.nbytes();
  m.num_elements = (uint64_t)t.numel();
  m.pinned = t.is_pinned() ? 1 : 0;
  m.requires_grad = t.requires_grad() ? 1 : 0;
  m.dtype = static_cast<int8_t>(t.scalar_type());
  m.device_index = static_cast<int8_t>(t.device().index());
  m.device_type = static_cast<int8_t>(t.device().type());
  m.layout = static_cast<int8_t>(t.layout());
  m.num_file_chunks = num_file_chunks;
  m.exp_file_offsets.assign(num_file_chunks, 0);
  m.compressed_sizes.assign(num_file_chunks, 0);
  m.original_sizes.assign(num_file_chunks, 0);
  return m;
}

class PrefetchHandle {
 public:
  PrefetchHandle(const std::string& offload_folder, const std::string& offload_file_name, const std::string& code_type,
                 const std::string& caching_algorithm, const double& device_memory_ratio,
                 const double& gpu_pool_ratio, double /*decompression_delay*/, double /*sm_io_delay*/,
                 int num_compute_threads, int num_file_chunks, int prefetcher_topk, int expert_topk,
                 size_t num_elements_per_expert, size_t num_tensors_per_expert, int num_expert_layers,
                 int num_experts, int lz4_accel, int lz4hc_level, int /*zstd_level*/, double state_margin,
                 bool /*bind_core*/)
      : s_(std::make_shared<Store>()) {
    if (num_file_chunks < 1) fail("num_file_chunks must be >= 1");
    if (code_type != "LZ4" && code_type != "LZ4HC") fail("CODE_TYPE '" + code_type + "' is not supported");
    Config& c = s_->cfg;
    c.code_type = code_type;
    c.caching_algorithm = caching_algorithm;
    c.device_memory_ratio = device_memory_ratio;
    c.gpu_pool_ratio = gpu_pool_ratio;
    c.state_margin = state_margin;
    c.num_compute_threads = std::max(1, num_compute_threads);
    c.num_file_chunks = num_file_chunks;
    c.prefetcher_topk = prefetcher_topk;
    c.expert_topk = std::max(1, expert_topk);
    c.num_elements_per_expert = num_elements_per_expert;
    c.num_tensors_per_expert = num_tensors_per_expert;
    c.num_expert_layers = std::max(1, num_expert_layers);
    c.num_experts = std::max(1, num_experts);
    c.lz4_accel = lz4_accel;
    c.lz4hc_level = lz4hc_level;
    s_->prefix = offload_folder;
    if (s_->prefix.empty() || s_->prefix.back() != '/') s_->prefix += '/';
    struct stat st;
    if (::stat(s_->prefix.c_str(), &st) == 0 && !S_ISDIR(st.st_mode)) fail(s_->prefix + " is not a directory");
    if (::stat(s_->prefix.c_str(), &st) != 0 && ::mkdir(s_->prefix.c_str(), 0777) != 0)
      fail("cannot create " + s_->prefix);
    s_->file.path = s_->prefix + offload_file_name;
    const std::string ip = s_->prefix + kIndexName;
    if (::access(ip.c_str(), F_OK) == 0) {
      s_->index.deserialize(read_file(ip));
      s_->index_loaded = true;
    }
    g_store = s_;
  }

  void open_offload_file() {
    std::lock_guard<std::mutex> g(s_->mu);
    s_->file.open_read();
  }

  void offload(uint32_t tensor_id, torch::Tensor& tensor,
               const std::vector<py::array_t<uint8_t, py::array::c_style | py::array::forcecast>>& exponents_chunks,
               const py::array_t<uint8_t, py::array::c_style | py::array::forcecast>& sign_mantissa, bool is_sparse) {
    ChunkArrays a = view_arrays(exponents_chunks, sign_mantissa);
    torch::Tensor host = is_sparse ? torch::Tensor() : tensor.detach().contiguous().cpu();
    {
      py::gil_scoped_release nogil;
      std::lock_guard<std::mutex> g(s_->mu);
      if (s_->index.has(tensor_id)) fail("tensor " + std::to_string(tensor_id) + " is offloaded twice");
      Meta m = meta_of(tensor_id, tensor, s_->cfg.num_file_chunks);
      if (is_sparse)
        store_sparse(m, a);
      else
        m.sm_file_offset = s_->file.append(host.data_ptr(), host.nbytes());
      s_->index.insert(tensor_id, std::move(m));
      write_file(s_->prefix + kIndexName, s_->index.serialize());
    }
  }

  void batch_offload(const std::vector<uint32_t> tensor_ids, std::vector<torch::Tensor>& tensors,
                     const std::vector<std::vector<py::array_t<uint8_t, py::array::c_style | py::array::forcecast>>>&
                         batch_exponents_chunks,
                     const std::vector<py::array_t<uint8_t, py::array::c_style | py::array::forcecast>>&
                         batch_sign_mantissa) {
    const size_t n = tensor_ids.size();
    if (tensors.size() != n || batch_exponents_chunks.size() != n || batch_sign_mantissa.size() != n)
      fail("batch_offload: argument lists differ in length");
    std::vector<ChunkArrays> arrays;
    for (size_t i = 0; i < n; ++i) arrays.push_back(view_arrays(batch_exponents_chunks[i], batch_sign_mantissa[i]));
    py::gil_scoped_release nogil;
    std::lock_guard<std::mutex> g(s_->mu);
    for (size_t i = 0; i < n; ++i)
      if (s_->index.has(tensor_ids[i])) fail("tensor " + std::to_string(tensor_ids[i]) + " is offloaded twice");
    std::vector<std::vector<uint8_t>> gpu_blocks;   // every chunk of the batch, in order
    const bool gpu = s_->cfg.gpu_encode && s_->cfg.code_type == "LZ4HC";
    if (gpu) {
      std::vector<std::pair<const uint8_t*, size_t>> all;
      for (auto& a : arrays) all.insert(all.end(), a.chunks.begin(), a.chunks.end());
      gpu_blocks = gpu_compress_chunks(all, s_->cfg.gpu_encode_attempts);
    }
    size_t next = 0;
    for (size_t i = 0; i < n; ++i) {
      Meta m = meta_of(tensor_ids[i], tensors[i], s_->cfg.num_file_chunks);
      store_sparse(m, arrays[i], gpu ? &gpu_blocks[next] : nullptr);
      next += arrays[i].chunks.size();
      s_->index.insert(tensor_ids[i], std::move(m));
    }
    write_file(s_->prefix + kIndexName, s_->index.serialize());
  }

  // Extension (no counterpart in the reference): batch_offload encodes LZ4HC
  // chunks on the GPU, trying `attempts` hash-chain candidates per position
  // (256, as LZ4HC level 9).  The blocks are valid LZ4 blocks but not liblz4's
  // bytes; the file layout and the index are unchanged.
  void set_gpu_encode(bool on, int attempts) {
    if (attempts < 1 || attempts > 65536) fail("set_gpu_encode: attempts outside [1, 65536]");
    std::lock_guard<std::mutex> g(s_->mu);
    s_->cfg.gpu_encode = on;
    s_->cfg.gpu_encode_attempts = attempts;
  }

  void register_tensor(torch::Tensor& tensor, uint32_t tensor_id) {
    std::lock_guard<std::mutex> g(s_->mu);
    s_->tensors[tensor_id] = tensor;
    s_->ptr_to_id[reinterpret_cast<uintptr_t>(tensor.data_ptr())] = tensor_id;
  }

  uint32_t begin(uint64_t /*request_id*/, torch::Tensor& tensor) {
    const uintptr_t old = reinterpret_cast<uintptr_t>(tensor.data_ptr());
    uint32_t id;
    Meta m;
    {
      std::lock_guard<std::mutex> g(s_->mu);
      id = id_of(old);
      m = s_->index.at(id);
    }
    torch::Tensor t = m.sparse() ? decode_tensor(*s_, m) : read_dense(*s_, m);
    if (t.scalar_type() != tensor.scalar_type()) t = t.to(tensor.scalar_type());
    tensor.set_data(t);
    remap(old, reinterpret_cast<uintptr_t>(tensor.data_ptr()));
    return id;
  }

  void end(uint64_t /*request_id*/, torch::Tensor& tensor) {
    const uintptr_t old = reinterpret_cast<uintptr_t>(tensor.data_ptr());
    tensor.set_data(torch::zeros({1}, torch::TensorOptions().dtype(tensor.scalar_type())));
    remap(old, reinterpret_cast<uintptr_t>(tensor.data_ptr()));
  }

  void set_topology(const std::vector<std::tuple<std::string, std::vector<std::vector<uint32_t>>>>& topology) {
    std::lock_guard<std::mutex> g(s_->mu);
    s_->topology = topology;
  }

  void update_tensor_map(uint64_t old_ptr, uint64_t new_ptr) { remap(old_ptr, new_ptr); }

  bool is_tensor_offloaded(uint32_t tensor_id) {
    std::lock_guard<std::mutex> g(s_->mu);
    return s_->index.has(tensor_id);
  }

  bool is_tensor_index_initialized() const { return s_->index_loaded; }

  int get_node_default_device(std::vector<uint32_t> /*tensor_ids*/) const { return c10::cuda::current_device(); }

  void fetch_tensors(uint64_t /*request_id*/, const std::vector<uint32_t>& ids) {
    for (uint32_t id : ids) {
      Meta m;
      torch::Tensor reg;
      {
        std::lock_guard<std::mutex> g(s_->mu);
        m = s_->index.at(id);
        auto it = s_->tensors.find(id);
        if (it == s_->tensors.end()) fail("tensor " + std::to_string(id) + " is not registered");
        reg = it->second;
      }
      if (m.sparse()) fail("fetch_tensors is for dense tensors; tensor " + std::to_string(id) + " is an expert tensor");
      const uintptr_t old = reinterpret_cast<uintptr_t>(reg.data_ptr());
      if (reg.is_cuda()) continue;
      reg.set_data(read_dense(*s_, m));
      remap(old, reinterpret_cast<uintptr_t>(reg.data_ptr()));
    }
  }

  void reset_access_counts() {
    std::vector<std::function<void()>> fs;
    {
      std::lock_guard<std::mutex> g(s_->mu);
      fs = s_->on_reset_counts;
    }
    for (auto& f : fs) f();
  }

 private:
  std::shared_ptr<Store> s_;

  uint32_t id_of(uintptr_t p) const {
    auto it = s_->ptr_to_id.find(p);
    if (it == s_->ptr_to_id.end()) fail("tensor is not registered");
    return it->second;
  }
  void remap(uintptr_t old_ptr, uintptr_t new_ptr) {
    std::lock_guard<std::mutex> g(s_->mu);
    auto it = s_->ptr_to_id.find(old_ptr);
    if (it == s_->ptr_to_id.end()) return;
    const uint32_t id = it->second;
    s_->ptr_to_id.erase(it);
    s_->ptr_to_id[new_ptr] = id;
  }
  // Compress the chunks on up to num_compute_threads threads, then append
  // chunk by chunk and the sign+mantissa plane (PipelineCompress order).
  // blocks: the chunks' LZ4 blocks when already encoded (GPU path), else null
  void store_sparse(Meta& m, const ChunkArrays& a, const std::vector<uint8_t>* pre = nullptr) {
    const int n = (int)a.chunks.size();
    if (n != m.num_file_chunks)
      fail("tensor " + std::to_string(m.id) + ": " + std::to_string(n) + " exponent chunks, num_file_chunks = " +
           std::to_string(m.num_file_chunks));
    uint64_t total = 0;
    for (auto& c : a.chunks) total += c.second;
    if (total != m.num_elements || a.sm_size != m.num_elements)
      fail("tensor " + std::to_string(m.id) + ": planes do not hold num_elements bytes");
    std::vector<std::vector<uint8_t>> blocks(n);
    if (pre) {
      for (int c = 0; c < n; ++c) blocks[c] = pre[c];
    } else {
      std::vector<std::future<void>> jobs;
      const int threads = std::min(n, s_->cfg.num_compute_threads);
      for (int w = 0; w < threads; ++w)
        jobs.push_back(std::async(std::launch::async, [&, w] {
          for (int c = w; c < n; c += threads) blocks[c] = compress_chunk(s_->cfg, a.chunks[c].first, a.chunks[c].second);
        }));
      for (auto& j : jobs) j.get();
    }
    for (int c = 0; c < n; ++c) {
      m.original_sizes[c] = a.chunks[c].second;
      m.compressed_sizes[c] = blocks[c].size();
      m.exp_file_offsets[c] = s_->file.append(blocks[c].data(), blocks[c].size());
    }
    m.sm_size = a.sm_size;
    m.sm_file_offset = s_->file.append(a.sm, a.sm_size);
  }
};

// ---------------------------------------------------------------------------
// expert_dispatcher
// ---------------------------------------------------------------------------
int cache_policy_of(const std::string& name) {
  if (name == "ZipMoE") return ZMOE_CACHE_ZIPMOE;
  if (name == "LFU") return ZMOE_CACHE_LFU;
  if (name == "LRU" || name == "Marking") return ZMOE_CACHE_LRU;   // Marking: evicts among unmarked, LRU order
  if (name == "FIFO") return ZMOE_CACHE_FIFO;
  fail("caching_algorithm '" + name + "' is not supported");
}

struct LayerEngine {
  zmoe_layer* L = nullptr;
  int E = 0, H = 0, I = 0, topk = 1, max_tokens = 0;
  ~LayerEngine() {
    if (L) zmoe_layer_destroy(L);
  }
};

class Dispatcher {
 public:
  using Result = std::tuple<torch::Tensor, int, int, int>;

  Dispatcher(int num_experts, int num_layers, int expert_type, int dtype)
      : E_(num_experts), layers_(num_layers), kind_(expert_type) {
    if (num_experts < 1 || num_layers < 1) fail("expert_dispatcher: num_experts and num_layers must be >= 1");
    if (expert_type != 0 && expert_type != 1) fail("expert_dispatcher: expert_type must be 0 (SwiGLU) or 1 (ReLU)");
    if (dtype != 0) fail("expert_dispatcher: only dtype 0 (BF16) is supported");
    ids_.assign(num_layers, std::vector<std::vector<uint32_t>>(num_experts));
    engines_.resize(num_layers);
    store_ = store_or_fail();
    std::weak_ptr<int> alive = alive_;
    auto* self = this;
    std::lock_guard<std::mutex> g(store_->mu);
    store_->on_reset_counts.push_back([alive, self] {
      if (alive.expired()) return;
      for (auto& e : self->engines_)
        if (e) zmoe_layer_reset_access_counts(e->L);
    });
  }

  void register_expert(int layer, int expert, const std::vector<uint32_t>& tensor_ids) {
    check_ids(layer, expert);
    const size_t want = kind_ == 0 ? 3 : 2;
    if (tensor_ids.size() != want)
      fail("register_expert: expected " + std::to_string(want) + " tensor ids, got " + std::to_string(tensor_ids.size()));
    ids_[layer][expert] = tensor_ids;
  }

  torch::Tensor obtain_tensor(int layer, int expert, int tensor_idx) {
    check_ids(layer, expert);
    const auto& ids = ids_[layer][expert];
    if (tensor_idx < 0 || tensor_idx >= (int)ids.size()) fail("obtain_tensor: tensor index out of range");
    Meta m;
    {
      std::lock_guard<std::mutex> g(store_->mu);
      m = store_->index.at(ids[tensor_idx]);
    }
    return decode_tensor(*store_, m);
  }

  void set_inputs(torch::Tensor hidden, torch::Tensor router_mask) {
    hidden_ = hidden.clone();
    mask_ = router_mask.clone();
  }

  void set_expected_queue(int n) { expected_ = n; }

  void enqueue_expert(int layer, int expert, int num_tokens) {
    check_ids(layer, expert);
    queue_.push_back({layer, expert, num_tokens});
  }

  void enqueue_prefetch(int layer, int expert) {
    check_ids(layer, expert);
    prefetch_.push_back({layer, expert});
  }

  void submit_prefetch(int layer, int expert, double /*priority*/) {
    check_ids(layer, expert);
    prefetch_.push_back({layer, expert});
    run_prefetch();
  }

  void ops_schedule() {
    run_prefetch();
    if (queue_.empty()) return;
    if (!hidden_.defined() || !mask_.defined()) fail("ops_schedule: set_inputs was not called");
    const c10::cuda::CUDAGuard guard(hidden_.device());
    torch::Tensor x = hidden_.reshape({-1, hidden_.size(-1)});
    if (!x.is_cuda()) x = x.to(torch::Device(torch::kCUDA, c10::cuda::current_device()));
    x = x.to(torch::kBFloat16).contiguous();
    const int64_t T = x.size(0), H = x.size(1);
    torch::Tensor mask = mask_.reshape({T, -1}).to(torch::kCPU).to(torch::kInt32).contiguous();
    if (mask.size(1) != E_) fail("router_mask has " + std::to_string(mask.size(1)) + " experts, expected " + std::to_string(E_));
    const int32_t* mk = mask.data_ptr<int32_t>();
    // per layer, in enqueue order
    std::vector<int> layers_seen;
    for (auto& q : queue_)
      if (std::find(layers_seen.begin(), layers_seen.end(), q.layer) == layers_seen.end()) layers_seen.push_back(q.layer);
    for (int layer : layers_seen) {
      std::vector<char> want(E_, 0);
      for (auto& q : queue_)
        if (q.layer == layer) want[q.expert] = 1;
      std::vector<int32_t> counts(E_, 0), index;
      std::vector<std::vector<int32_t>> toks(E_);
      for (int e = 0; e < E_; ++e) {
        if (!want[e]) continue;
        for (int64_t t = 0; t < T; ++t)
          if (mk[t * E_ + e] != 0) toks[e].push_back((int32_t)t);
        counts[e] = (int32_t)toks[e].size();
        index.insert(index.end(), toks[e].begin(), toks[e].end());
      }
      const int rows = (int)index.size();
      LayerEngine& eng = engine(layer, H, rows);
      std::vector<int32_t> cached(E_);
      int nc = 0;
      check(zmoe_layer_cached_experts(eng.L, cached.data(), E_, &nc), "zmoe_layer_cached_experts");
      std::vector<char> hit(E_, 0);
      for (int i = 0; i < nc; ++i) hit[cached[i]] = 1;
      torch::Tensor y;
      if (rows > 0) {
        auto idx = torch::from_blob(index.data(), {rows}, torch::kInt32).to(x.device());
        auto xg = torch::empty({rows, H}, x.options());
        check(zmoe_gather_rows(x.data_ptr(), idx.data_ptr<int32_t>(), rows, (int)(H * 2), xg.data_ptr(),
                               current_stream()),
              "zmoe_gather_rows");
        auto yf = torch::empty({rows, H}, x.options().dtype(torch::kBFloat16));
        check(zmoe_layer_experts(eng.L, reinterpret_cast<const uint16_t*>(xg.data_ptr()), counts.data(), rows,
                                 reinterpret_cast<uint16_t*>(yf.data_ptr()), current_stream()),
              "zmoe_layer_experts");
        y = yf;                                      // BF16, as the reference's experts return it
      }
      std::vector<int64_t> start(E_ + 1, 0);
      for (int e = 0; e < E_; ++e) start[e + 1] = start[e] + counts[e];
      auto dev = hidden_.device();
      for (auto& q : queue_) {
        if (q.layer != layer) continue;
        torch::Tensor out = counts[q.expert] > 0 ? y.narrow(0, start[q.expert], counts[q.expert])
                                                 : torch::empty({0, H}, x.options());
        if (out.device() != dev) out = out.to(dev);
        results_.emplace_back(out, q.layer, q.expert, hit[q.expert] ? 1 : 0);
      }
    }
    queue_.clear();
  }

  std::vector<Result> wait_expert() {
    if (!queue_.empty()) ops_schedule();
    if (expected_ > 0 && (int)results_.size() != expected_)
      fail("wait_expert: " + std::to_string(results_.size()) + " results, set_expected_queue said " +
           std::to_string(expected_));
    cuda_check(cudaStreamSynchronize(current_stream()), "wait_expert");
    std::vector<Result> out;
    out.swap(results_);
    expected_ = 0;
    return out;
  }

 private:
  struct Req {
    int layer, expert, tokens;
  };
  int E_, layers_, kind_;
  std::vector<std::vector<std::vector<uint32_t>>> ids_;   // [layer][expert] -> tensor ids
  std::vector<std::unique_ptr<LayerEngine>> engines_;
  std::shared_ptr<Store> store_;
  std::shared_ptr<int> alive_ = std::make_shared<int>(0);
  torch::Tensor hidden_, mask_;
  int expected_ = 0;
  std::vector<Req> queue_;
  std::vector<std::pair<int, int>> prefetch_;
  std::vector<Result> results_;

  void check_ids(int layer, int expert) const {
    if (layer < 0 || layer >= layers_) fail("layer " + std::to_string(layer) + " out of range");
    if (expert < 0 || expert >= E_) fail("expert " + std::to_string(expert) + " out of range");
  }

  void run_prefetch() {
    if (prefetch_.empty()) return;
    std::vector<std::pair<int, int>> todo;
    todo.swap(prefetch_);
    for (auto [layer, expert] : todo) {
      LayerEngine* eng = engines_[layer].get();
      if (!eng) eng = &engine(layer, 0, 0);
      int e = expert;
      check(zmoe_layer_prefetch(eng->L, &e, 1, current_stream()), "zmoe_layer_prefetch");
    }
  }

  // The layer's engine, created on first use from the offload file; rebuilt
  // (experts reloaded) when a call needs more rows than its workspace holds.
  LayerEngine& engine(int layer, int64_t H, int rows) {
    auto& slot = engines_[layer];
    if (slot && rows <= slot->max_tokens * slot->topk) return *slot;
    std::vector<std::vector<Meta>> metas(E_);
    {
      std::lock_guard<std::mutex> g(store_->mu);
      for (int e = 0; e < E_; ++e) {
        if (ids_[layer][e].empty()) fail("layer " + std::to_string(layer) + " expert " + std::to_string(e) + " is not registered");
        for (uint32_t id : ids_[layer][e]) metas[e].push_back(store_->index.at(id));
      }
    }
    const Meta& m0 = metas[0][0];
    if (m0.shape.size() != 2) fail("expert tensors must be 2-D");
    auto eng = std::make_unique<LayerEngine>();
    eng->E = E_;
    eng->I = (int)m0.shape[0];
    eng->H = (int)m0.shape[1];
    if (H > 0 && H != eng->H) fail("hidden size " + std::to_string(H) + " does not match the experts' " + std::to_string(eng->H));
    const Config& c = store_->cfg;
    eng->topk = std::max(1, std::min({c.expert_topk, E_, 8}));
    const int prev = slot ? slot->max_tokens : 0;
    eng->max_tokens = std::max({64, prev, 2 * ((rows + eng->topk - 1) / eng->topk)});
    cudaDeviceProp prop;
    cuda_check(cudaGetDeviceProperties(&prop, c10::cuda::current_device()), "cudaGetDeviceProperties");
    const double expert_bytes = (double)(kind_ == 0 ? 3 : 2) * eng->H * (double)eng->I * 2.0;
    const double pool = (double)prop.totalGlobalMem * c.device_memory_ratio * c.gpu_pool_ratio;
    int cache = (int)(pool / expert_bytes / c.num_expert_layers);
    cache = std::max(0, std::min(cache, E_));
    // the rest of the budget holds sign+mantissa planes (1 byte per element),
    // the reference's SM pool (runtime/cache_planning.py:71-88); the engine
    // uses it when its experts are stored in host memory
    const double sm_pool = (double)prop.totalGlobalMem * c.device_memory_ratio * (1.0 - c.gpu_pool_ratio);
    int sm = (int)(sm_pool / (expert_bytes / 2.0) / c.num_expert_layers);
    sm = std::max(0, std::min(sm, E_ - cache));
    zmoe_layer_config cfg{};
    cfg.hidden = eng->H;
    cfg.num_experts = E_;
    cfg.inter = eng->I;
    cfg.topk = eng->topk;
    cfg.kind = kind_;
    cfg.route_mode = kind_ == 1 ? ZMOE_ROUTE_SWITCH : ZMOE_ROUTE_DEEPSEEK;
    cfg.scaling = 1.0f;
    cfg.max_tokens = eng->max_tokens;
    cfg.cache_slots = cache;
    cfg.transient_slots = std::max(1, std::min(E_ - cache, 32));
    cfg.cache_policy = cache_policy_of(c.caching_algorithm);
    cfg.state_margin = c.state_margin;
    cfg.sm_slots = sm;
    check(zmoe_layer_create(&cfg, &eng->L), "zmoe_layer_create");
    for (int e = 0; e < E_; ++e)
      for (size_t t = 0; t < metas[e].size(); ++t) {
        const Meta& m = metas[e][t];
        HostPlanes p = read_planes(*store_, m);
        std::vector<const uint8_t*> ptrs;
        for (auto& b : p.blocks) ptrs.push_back(b.data());
        check(zmoe_layer_load_expert(eng->L, e, (int)t, ptrs.data(), p.block_sizes.data(), p.original_sizes.data(),
                                     (int)ptrs.size(), p.sm.data(), m.num_elements),
              "zmoe_layer_load_expert");
      }
    slot = std::move(eng);
    return *slot;
  }
};

}  // namespace zipmoe

PYBIND11_MODULE(ZipMoE, m) {
  using namespace zipmoe;
  m.doc() = "B200 expert path behind the reference's ZipMoE operator surface";
  py::class_<PrefetchHandle>(m, "zipmoe_prefetch_handle")
      .def(py::init<const std::string&, const std::string&, const std::string&, const std::string&, const double&,
                    const double&, double, double, int, int, int, int, size_t, size_t, int, int, int, int, int, double,
                    bool>(),
           py::arg("offload_folder"), py::arg("offload_file_name"), py::arg("CODE_TYPE"),
           py::arg("caching_algorithm"), py::arg("device_memory_ratio"), py::arg("gpu_pool_ratio"),
           py::arg("decompression_delay"), py::arg("sm_io_delay"), py::arg("num_compute_threads"),
           py::arg("num_file_chunks"), py::arg("prefetcher_topk"), py::arg("expert_topk"),
           py::arg("num_elements_per_expert"), py::arg("num_tensors_per_expert"), py::arg("num_expert_layers"),
           py::arg("num_experts"), py::arg("LZ4_accelerationLevel"), py::arg("LZ4HC_compressionLevel"),
           py::arg("ZSTD_compressionLevel"), py::arg("hyperparam_state_margin"), py::arg("bind_core"))
      .def("open_offload_file", &PrefetchHandle::open_offload_file,
           "Open the offloaded file after the offloading is completed.")
      .def("offload", &PrefetchHandle::offload, "Offload a tensor.")
      .def("batch_offload", &PrefetchHandle::batch_offload, "Offload tensors in a batch.")
      .def("set_gpu_encode", &PrefetchHandle::set_gpu_encode, py::arg("on"), py::arg("attempts") = 256,
           "Encode batch_offload's LZ4HC chunks on the GPU (extension).")
      .def("register", &PrefetchHandle::register_tensor, "Register a buffer under its tensor id.")
      .def("begin", &PrefetchHandle::begin, "Pre hook: materialise the tensor on the GPU; returns its id.")
      .def("end", &PrefetchHandle::end, "Post hook: release the tensor's device copy.")
      .def("set_topology", &PrefetchHandle::set_topology, "Set up the model topology.")
      .def("update_tensor_map", &PrefetchHandle::update_tensor_map, "Move a registered tensor to a new data pointer.")
      .def("is_tensor_offloaded", &PrefetchHandle::is_tensor_offloaded, "Check whether a tensor is offloaded.")
      .def("is_tensor_index_initialized", &PrefetchHandle::is_tensor_index_initialized,
           "Whether an index file was found when the handle was created.")
      .def("get_node_default_device", &PrefetchHandle::get_node_default_device,
           "Returns the device index of a given node.")
      .def("fetch_tensors", &PrefetchHandle::fetch_tensors, "Materialise dense tensors on the GPU.")
      .def("reset_access_counts", &PrefetchHandle::reset_access_counts,
           "Reset the per-expert access counts of every layer's cache.");

  py::class_<Dispatcher>(m, "expert_dispatcher")
      .def(py::init<int, int, int, int>(), py::arg("num_experts"), py::arg("num_layers"), py::arg("expert_type"),
           py::arg("dtype"))
      .def("register_expert", &Dispatcher::register_expert, "Register the experts.")
      .def("obtain_tensor", &Dispatcher::obtain_tensor, "Obtain the tensor for debugging.")
      .def("enqueue_expert", &Dispatcher::enqueue_expert, "Queue an expert of a layer for this forward.")
      .def("enqueue_prefetch", &Dispatcher::enqueue_prefetch, "Queue a prefetch (run at the next ops_schedule).")
      .def("submit_prefetch", &Dispatcher::submit_prefetch, "Decode an expert into the cache now.")
      .def("ops_schedule", &Dispatcher::ops_schedule, "Decode misses and run the queued experts.")
      .def("set_inputs", &Dispatcher::set_inputs, "Clone the hidden states and the router mask.")
      .def("set_expected_queue", &Dispatcher::set_expected_queue, "Number of results wait_expert returns.")
      .def("wait_expert", &Dispatcher::wait_expert, py::call_guard<py::gil_scoped_release>(),
           "Wait for the queued experts; returns [(output, layer, expert, hit)].");
}
