// .mojostream model files and lm_head_proto.bin -> a device model.
//
// Format (little-endian; src/streaming/mojostream.mojo:95-160, written by
// scripts/create_fake_model.py:194-281 and scripts/convert.py:359-414):
//   header   128 B: "MOJOSTRM", version, format tag, n_layers, hidden, kv_dim,
//            ffn_dim, n_heads, n_kv_heads (u32), n_tensors, dir_offset,
//            data_start (u64); format 2 adds at byte 64 "ENGR", version,
//            kv-shared layers, sliding kv_dim, full kv_dim, PLE dim, window
//   directory n_tensors x 32 B: layer, type (0 PLE, 1-7 Q K V O Gate Up Down),
//            rows, cols, scale (f32), flags, data offset (u64; 0 for PLE)
//   data     per tensor rows x cols/2 bytes of Q4, on 4096-byte boundaries
// The checks are the reference's ShapeGuard / TensorGuard
// (src/streaming/stream_runner.mojo:288-400), with layer-typed dims accepted
// for format 2.  Loading streams the data region through pinned host buffers,
// one per reader thread (preads in parallel, each overlapping the others'
// cudaMemcpyAsync: the double buffer of src/streaming/sparse_pin.mojo:136-330
// widened, and aimed at HBM once since the models fit), and hands device
// pointers to ms_model_create.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "ms_internal.h"
#include "ms_kernels.h"

namespace {

constexpr uint32_t kMagic = 0x4F4A4F4Du;  // "MOJO": the reference checks these 4 bytes
constexpr int kHeaderBytes = 128, kEntryBytes = 32, kPerLayer = 8;
constexpr uint64_t kPage = 4096;
constexpr int kMaxDim = 1 << 24;
enum { kPle = 0, kQ, kK, kV, kO, kGate, kUp, kDown };
const char* const kMatNames[8] = {"PLE", "Q", "K", "V", "O", "Gate", "Up", "Down"};

struct Entry {
  uint32_t layer, type, rows, cols;
  float scale;
  uint64_t offset;
};

struct FileView {
  int fd = -1;
  ms_file_info info{};
  std::vector<Entry> entries;
  std::vector<int> head_dim;  // per layer
  ms_status code = MS_OK;
  std::string err;
  FileView() = default;
  FileView(const FileView&) = delete;
  ~FileView() {
    if (fd >= 0) close(fd);
  }
  bool fail(ms_status s, const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    code = s;
    err = b;
    return false;
  }
};

uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}
uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  memcpy(&v, p, 8);
  return v;
}
float rdf(const uint8_t* p) {
  float v;
  memcpy(&v, p, 4);
  return v;
}

bool pread_all(int fd, void* dst, size_t n, uint64_t off) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  while (n) {
    const ssize_t r = pread(fd, d, n, (off_t)off);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    d += r;
    n -= (size_t)r;
    off += (uint64_t)r;
  }
  return true;
}

bool open_file(const char* path, FileView& f, uint64_t* size) {
  f.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f.fd < 0) return f.fail(MS_ERR_INVALID_ARG, "cannot open %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(f.fd, &st) != 0) return f.fail(MS_ERR_INVALID_ARG, "stat %s: %s", path, strerror(errno));
  *size = (uint64_t)st.st_size;
  return true;
}

// Header, ShapeGuard, directory, TensorGuard (stream_runner.mojo:172-400).
bool read_and_check(const char* path, FileView& f) {
  ms_file_info& I = f.info;
  if (!open_file(path, f, &I.file_size)) return false;
  if (I.file_size <= (uint64_t)kHeaderBytes)
    return f.fail(MS_ERR_SHAPE, "file too small: %llu bytes", (unsigned long long)I.file_size);
  uint8_t h[kHeaderBytes];
  if (!pread_all(f.fd, h, kHeaderBytes, 0)) return f.fail(MS_ERR_INVALID_ARG, "header read failed");
  if (rd32(h) != kMagic) return f.fail(MS_ERR_SHAPE, "invalid magic: not a .mojostream file");
  I.format_tag = (int)rd32(h + 12);
  const uint32_t u[6] = {rd32(h + 16), rd32(h + 20), rd32(h + 24), rd32(h + 28), rd32(h + 32), rd32(h + 36)};
  for (uint32_t v : u)
    if (v > (uint32_t)kMaxDim) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] header field %u out of range", v);
  I.n_layers = (int)u[0];
  I.hidden = (int)u[1];
  I.kv_dim = (int)u[2];
  I.ffn_dim = (int)u[3];
  I.n_heads = (int)u[4];
  I.n_kv_heads = (int)u[5];
  I.n_tensors = rd64(h + 40);
  I.data_start = rd64(h + 56);
  if (memcmp(h + 64, "ENGR", 4) == 0) {
    I.kv_shared_layers = (int)std::min<uint32_t>(rd32(h + 72), kMaxDim);
    I.sliding_kv_dim = (int)std::min<uint32_t>(rd32(h + 76), kMaxDim);
    I.full_kv_dim = (int)std::min<uint32_t>(rd32(h + 80), kMaxDim);
    I.ple_dim = (int)std::min<uint32_t>(rd32(h + 84), kMaxDim);
    I.sliding_window = (int)std::min<uint32_t>(rd32(h + 88), kMaxDim);
  }
  if (I.format_tag != 1 && I.format_tag != 2)
    return f.fail(MS_ERR_SHAPE, "format tag %d (1: gemma4_q4_rowmajor, 2: layer-typed)", I.format_tag);
  const bool typed = I.format_tag == 2;
  const int D = I.hidden, NH = I.n_heads, NKV = I.n_kv_heads, KVD = I.kv_dim, F = I.ffn_dim;

  // ShapeGuard (stream_runner.mojo:288-318)
  if (NH == 0) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] n_heads = 0");
  if (NKV == 0) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] n_kv_heads = 0");
  if (D % NH) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] hidden=%d not divisible by n_heads=%d", D, NH);
  if (NH % NKV)
    return f.fail(MS_ERR_SHAPE, "[ShapeGuard] n_heads=%d not divisible by n_kv_heads=%d", NH, NKV);
  if (!typed && KVD != NKV * (D / NH))
    return f.fail(MS_ERR_SHAPE, "[ShapeGuard] kv_dim=%d expected=%d (n_kv_heads x head_dim)", KVD,
                  NKV * (D / NH));
  if (typed && KVD % NKV)  // head_dim may differ from hidden / n_heads (E4B)
    return f.fail(MS_ERR_SHAPE, "[ShapeGuard] kv_dim=%d not divisible by n_kv_heads=%d", KVD, NKV);
  if (I.n_layers <= 0) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] n_layers <= 0");
  if (F <= 0) return f.fail(MS_ERR_SHAPE, "[ShapeGuard] ffn_dim <= 0");
  if (I.n_tensors != (uint64_t)I.n_layers * kPerLayer)
    return f.fail(MS_ERR_SHAPE, "[ShapeGuard] n_tensors=%llu expected=%d (n_layers x %d)",
                  (unsigned long long)I.n_tensors, I.n_layers * kPerLayer, kPerLayer);

  // directory
  const uint64_t dir_bytes = I.n_tensors * kEntryBytes;
  if (kHeaderBytes + dir_bytes > I.file_size)
    return f.fail(MS_ERR_SHAPE, "directory (%llu entries) runs past the file end",
                  (unsigned long long)I.n_tensors);
  std::vector<uint8_t> dir(dir_bytes);
  if (!pread_all(f.fd, dir.data(), dir_bytes, kHeaderBytes))
    return f.fail(MS_ERR_INVALID_ARG, "directory read failed");
  f.entries.resize(I.n_tensors);
  for (uint64_t i = 0; i < I.n_tensors; ++i) {
    const uint8_t* e = dir.data() + i * kEntryBytes;
    f.entries[i] = Entry{rd32(e), rd32(e + 4), rd32(e + 8), rd32(e + 12), rdf(e + 16), rd64(e + 24)};
  }

  // per-layer head_dim: format 1 hidden / n_heads; format 2 from Q's columns
  f.head_dim.assign(I.n_layers, D / NH);
  for (int l = 0; l < I.n_layers && typed; ++l) {
    const Entry& q = f.entries[(size_t)l * kPerLayer + kQ];
    if (q.cols == 0 || q.cols % NH)
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Layer %d Q: cols=%u not a multiple of n_heads=%d", l,
                    q.cols, NH);
    const int hd = (int)(q.cols / NH);
    if ((I.sliding_kv_dim || I.full_kv_dim) && NKV * hd != I.sliding_kv_dim && NKV * hd != I.full_kv_dim)
      return f.fail(MS_ERR_SHAPE,
                    "[TensorGuard] Layer %d: head_dim %d gives kv_dim %d, neither sliding %d nor full %d",
                    l, hd, NKV * hd, I.sliding_kv_dim, I.full_kv_dim);
    f.head_dim[l] = hd;
  }

  // TensorGuard (stream_runner.mojo:320-400)
  uint64_t data_end = I.data_start;
  for (uint64_t i = 0; i < I.n_tensors; ++i) {
    const Entry& e = f.entries[i];
    const int layer = (int)(i / kPerLayer), type = (int)(i % kPerLayer);
    const int q = NH * f.head_dim[layer], kv = NKV * f.head_dim[layer];
    const uint32_t exp_r[8] = {1, (uint32_t)D, (uint32_t)D, (uint32_t)D, (uint32_t)q, (uint32_t)D, (uint32_t)D, (uint32_t)F};
    const uint32_t exp_c[8] = {0, (uint32_t)q, (uint32_t)kv, (uint32_t)kv, (uint32_t)D, (uint32_t)F, (uint32_t)F, (uint32_t)D};
    const char* nm = kMatNames[type];
    if (e.layer != (uint32_t)layer)
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: layer_id=%u expected=%d",
                    (unsigned long long)i, layer, nm, e.layer, layer);
    if (e.type != (uint32_t)type)
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: mat_type=%u expected=%d",
                    (unsigned long long)i, layer, nm, e.type, type);
    if (e.rows != exp_r[type])
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: rows=%u expected=%u",
                    (unsigned long long)i, layer, nm, e.rows, exp_r[type]);
    if (e.cols != exp_c[type])
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: cols=%u expected=%u",
                    (unsigned long long)i, layer, nm, e.cols, exp_c[type]);
    if (!(e.scale > 0.f))
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: scale=%g <= 0",
                    (unsigned long long)i, layer, nm, (double)e.scale);
    if (type == kPle) continue;
    if (e.offset % kPage)
      return f.fail(MS_ERR_SHAPE, "[TensorGuard] Tensor[%llu] Layer %d %s: offset=%llu not 4096-aligned",
                    (unsigned long long)i, layer, nm, (unsigned long long)e.offset);
    const uint64_t bytes = (uint64_t)e.rows * (e.cols / 2);
    // (written so that no sum can wrap: offsets are 64-bit values from the file)
    if (e.offset < I.data_start || e.offset > I.file_size || bytes > I.file_size - e.offset)
      return f.fail(MS_ERR_SHAPE,
                    "[TensorGuard] Tensor[%llu] Layer %d %s: offset=%llu + size=%llu outside the data "
                    "region [%llu, %llu)",
                    (unsigned long long)i, layer, nm, (unsigned long long)e.offset,
                    (unsigned long long)bytes, (unsigned long long)I.data_start,
                    (unsigned long long)I.file_size);
    data_end = std::max(data_end, e.offset + bytes);
  }
  I.data_end = data_end;
  return true;
}

// Reader threads, each with its own pinned buffer: a thread preads its next
// chunk while the copies of the others' (and its own previous one, until its
// event completes) run on the stream, so disk / page-cache reads proceed in
// parallel and overlap the host-to-device DMA.
struct Staging {
  std::vector<uint8_t*> pin;
  std::vector<cudaEvent_t> ev;
  size_t bytes = 0;
  bool init(int n, size_t b) {
    bytes = b;
    pin.assign(n, nullptr);
    ev.assign(n, nullptr);
    for (int i = 0; i < n; ++i) {
      if (cudaHostAlloc((void**)&pin[i], b, cudaHostAllocDefault) != cudaSuccess) return false;
      if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) return false;
    }
    return true;
  }
  ~Staging() {
    for (size_t i = 0; i < pin.size(); ++i) {
      if (ev[i]) cudaEventSynchronize(ev[i]), cudaEventDestroy(ev[i]);
      if (pin[i]) cudaFreeHost(pin[i]);
    }
  }
};

bool stream_to_device(int fd, uint64_t off, uint64_t n, uint8_t* dev, Staging& S, cudaStream_t s,
                      int device, std::string& err) {
  const int T = (int)S.pin.size();
  const uint64_t chunks = (n + S.bytes - 1) / S.bytes;
  std::atomic<bool> bad{false};
  std::mutex mu;
  auto worker = [&](int t) {
    cudaSetDevice(device);
    for (uint64_t k = t; k < chunks && !bad.load(); k += T) {
      cudaEventSynchronize(S.ev[t]);  // this thread's previous copy has finished
      const uint64_t at = k * S.bytes;
      const size_t len = (size_t)std::min<uint64_t>(S.bytes, n - at);
      std::string e;
      if (!pread_all(fd, S.pin[t], len, off + at))
        e = "read failed at offset " + std::to_string(off + at);
      else if (cudaMemcpyAsync(dev + at, S.pin[t], len, cudaMemcpyHostToDevice, s) != cudaSuccess ||
               cudaEventRecord(S.ev[t], s) != cudaSuccess)
        e = std::string("host-to-device copy: ") + cudaGetErrorString(cudaGetLastError());
      if (!e.empty()) {
        std::lock_guard<std::mutex> g(mu);
        if (!bad.exchange(true)) err = e;
        return;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < T && (uint64_t)t < chunks; ++t) pool.emplace_back(worker, t);
  worker(0);
  for (auto& th : pool) th.join();
  const cudaError_t e = cudaStreamSynchronize(s);
  if (!bad.load() && e != cudaSuccess) {
    err = std::string("host-to-device copy: ") + cudaGetErrorString(e);
    return false;
  }
  return !bad.load();
}

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

}  // namespace

extern "C" ms_status ms_file_check(const char* path, ms_file_info* info, char* err, size_t err_bytes) {
  if (err && err_bytes) err[0] = 0;
  if (!path) return MS_ERR_INVALID_ARG;
  FileView f;
  const bool ok = read_and_check(path, f);
  if (info) *info = f.info;
  if (!ok && err && err_bytes) snprintf(err, err_bytes, "%s", f.err.c_str());
  return ok ? MS_OK : f.code;
}

extern "C" ms_status ms_model_load(ms_ctx* c, const char* path, const char* lm_head_path,
                                   const ms_load_opts* opts_in, ms_model** out) {
  if (!c || !path || !out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  ms_load_opts o{};
  if (opts_in) o = *opts_in;
  FileView f;
  if (!read_and_check(path, f)) return ms_fail_(c, f.code, f.err.c_str());
  const ms_file_info& I = f.info;
  const bool typed = I.format_tag == 2;
  const int full_every = o.full_every > 0 ? o.full_every : (typed ? 6 : 1);
  const int window = o.window > 0 ? o.window : I.sliding_window;
  const float slide_theta = o.slide_theta > 0.f ? o.slide_theta : 1e4f;
  const float full_theta = o.full_theta > 0.f ? o.full_theta : (typed ? 1e6f : slide_theta);
  const int max_rows = o.max_rows > 0 ? o.max_rows : 64;
  const size_t staging = o.staging_bytes ? o.staging_bytes : ((size_t)32 << 20);
  const int readers = (int)std::max(1u, std::min(8u, std::thread::hardware_concurrency() / 2));
  char msg[512];

  // layer table (what the file does not say comes from the options)
  std::vector<ms_layer_desc> L(I.n_layers);
  for (int l = 0; l < I.n_layers; ++l) {
    const int hd = f.head_dim[l];
    const bool full = (l + 1) % full_every == 0;
    if (typed && I.sliding_kv_dim && I.full_kv_dim && I.sliding_kv_dim != I.full_kv_dim &&
        I.n_kv_heads * hd != (full ? I.full_kv_dim : I.sliding_kv_dim)) {
      snprintf(msg, sizeof msg,
               "layer %d is %s attention by full_every=%d, but its K has %d columns (%s kv_dim %d)", l,
               full ? "full" : "sliding", full_every, I.n_kv_heads * hd, full ? "full" : "sliding",
               full ? I.full_kv_dim : I.sliding_kv_dim);
      return ms_fail_(c, MS_ERR_SHAPE, msg);
    }
    if (!full && window <= 0) {
      snprintf(msg, sizeof msg, "layer %d is sliding but neither the file nor the options give a window", l);
      return ms_fail_(c, MS_ERR_SHAPE, msg);
    }
    ms_layer_desc& d = L[l];
    memset(&d, 0, sizeof d);
    d.head_dim = hd;
    d.n_heads = I.n_heads;
    d.n_kv_heads = I.n_kv_heads;
    d.window = full ? 0 : window;
    const int fr = o.full_rotary > 0 ? o.full_rotary : (typed ? 128 : hd);
    d.rotary_dims = full ? std::min(fr, hd) : hd;
    d.ffn_dim = I.ffn_dim;
    d.rope_theta = full ? full_theta : slide_theta;
    d.ple = f.entries[(size_t)l * kPerLayer + kPle].scale;
    for (int j = 0; j < 7; ++j) d.scale[j] = f.entries[(size_t)l * kPerLayer + 1 + j].scale;
  }

  cudaSetDevice(ms_device_(c));
  cudaStream_t s = ms_stream_(c);
  Staging S;
  if (!S.init(readers, staging)) return ms_fail_(c, MS_ERR_OOM, "pinned staging buffers");
  const auto t0 = std::chrono::steady_clock::now();
  uint64_t moved = 0;
  std::string err;

  // layer data: [data_start, data_end) in one device block
  DevBuf raw;
  const uint64_t span = I.data_end - I.data_start;
  if (cudaMalloc(&raw.p, span ? span : 16) != cudaSuccess) {
    cudaGetLastError();
    return ms_fail_(c, MS_ERR_OOM, "device buffer for the layer data");
  }
  if (!stream_to_device(f.fd, I.data_start, span, (uint8_t*)raw.p, S, s, ms_device_(c), err))
    return ms_fail_(c, MS_ERR_CUDA, err.c_str());
  moved += span;
  for (int l = 0; l < I.n_layers; ++l)
    for (int j = 0; j < 7; ++j)
      L[l].w[j] = (const uint8_t*)raw.p + (f.entries[(size_t)l * kPerLayer + 1 + j].offset - I.data_start);

  // lm_head_proto.bin (load_lm_head, lm_head.mojo:61-116)
  ms_model_desc desc{};
  desc.hidden = I.hidden;
  desc.n_layers = I.n_layers;
  desc.layers = L.data();
  desc.max_rows = max_rows;
  DevBuf lm, lmq, bos_dev;
  std::vector<float> gamma, bos;
  if (lm_head_path) {
    FileView g;
    uint64_t size = 0;
    if (!open_file(lm_head_path, g, &size)) return ms_fail_(c, g.code, g.err.c_str());
    const uint64_t D = (uint64_t)I.hidden;
    uint8_t h[12] = {0};
    if (size < 8 || !pread_all(g.fd, h, std::min<uint64_t>(12, size), 0))
      return ms_fail_(c, MS_ERR_SHAPE, "lm_head file: header read failed");
    const uint64_t V = rd32(h);
    const float q_scale = rdf(h + 4);
    // v2 is recognised by its size, as the reference does (lm_head.mojo:77-79)
    const bool v2 = size >= 12 + 8 * D + 4 * D * V;
    if (V == 0 || V % 4 || V > (1u << 26)) {
      snprintf(msg, sizeof msg, "lm_head file: vocab %llu (needs a multiple of 4)", (unsigned long long)V);
      return ms_fail_(c, MS_ERR_SHAPE, msg);
    }
    if (v2 && rd32(h + 8) != 2) return ms_fail_(c, MS_ERR_SHAPE, "lm_head file: version field is not 2");
    if (!v2 && size < 8 + 4 * D + D * V / 2) {
      snprintf(msg, sizeof msg, "lm_head file: %llu bytes, below v1 (%llu) and v2 (%llu) for hidden %llu",
               (unsigned long long)size, (unsigned long long)(8 + 4 * D + D * V / 2),
               (unsigned long long)(12 + 8 * D + 4 * D * V), (unsigned long long)D);
      return ms_fail_(c, MS_ERR_SHAPE, msg);
    }
    const uint64_t bos_off = v2 ? 12 : 8;
    bos.resize(D);
    if (!pread_all(g.fd, bos.data(), D * 4, bos_off)) return ms_fail_(c, MS_ERR_SHAPE, "lm_head file: BOS read");
    if (v2) {
      gamma.resize(D);
      if (!pread_all(g.fd, gamma.data(), D * 4, bos_off + 4 * D))
        return ms_fail_(c, MS_ERR_SHAPE, "lm_head file: gamma read");
    }
    if (cudaMalloc(&lm.p, D * V * 4) != cudaSuccess) {
      cudaGetLastError();
      return ms_fail_(c, MS_ERR_OOM, "device buffer for the lm_head");
    }
    if (v2) {
      if (!stream_to_device(g.fd, 12 + 8 * D, D * V * 4, (uint8_t*)lm.p, S, s, ms_device_(c), err))
        return ms_fail_(c, MS_ERR_CUDA, err.c_str());
      moved += D * V * 4;
    } else {  // Q4 [D][V/2]: expanded to the fp32 values (nibble - 8) * scale
      if (cudaMalloc(&lmq.p, D * V / 2) != cudaSuccess) {
        cudaGetLastError();
        return ms_fail_(c, MS_ERR_OOM, "device buffer for the Q4 lm_head");
      }
      if (!stream_to_device(g.fd, 8 + 4 * D, D * V / 2, (uint8_t*)lmq.p, S, s, ms_device_(c), err))
        return ms_fail_(c, MS_ERR_CUDA, err.c_str());
      moved += D * V / 2;
      if (ms::launch_dequant_q4_f32((float*)lm.p, (const uint8_t*)lmq.p, D * V / 2, q_scale, s) !=
              cudaSuccess ||
          cudaStreamSynchronize(s) != cudaSuccess)
        return ms_fail_(c, MS_ERR_CUDA, "lm_head dequant");
    }
    if (cudaMalloc(&bos_dev.p, D * 4) != cudaSuccess ||
        cudaMemcpy(bos_dev.p, bos.data(), D * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      return ms_fail_(c, MS_ERR_OOM, "BOS embedding");
    }
    desc.vocab = (int)V;
    desc.lm_head = (const float*)lm.p;
    desc.final_gamma = gamma.empty() ? nullptr : gamma.data();  // v1: gamma 1
  }
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  ms_set_load_stats_(c, secs, moved);

  ms_model* m = nullptr;
  const ms_status st = ms_model_create(c, &desc, &m);
  if (st != MS_OK) return st;
  if (lm_head_path) {
    // apply_bos_embedding (lm_head.mojo:133-143): the BOS token (id 2) embeds
    // as the file's BOS vector
    const ms_status sb = ms_model_set_bos_(c, m, (const float*)bos_dev.p, 2);
    if (sb != MS_OK) {
      ms_model_destroy(c, m);
      return sb;
    }
  }
  *out = m;
  return MS_OK;
}
