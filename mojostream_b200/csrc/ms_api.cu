// ms_api.cu -- the C-ABI of libmojostream_cuda.so (include/mojostream_cuda.h):
// contexts, weight upload + repack, the paged KV cache, layer orchestration,
// CUDA-graph decode loop.
//
// Per layer the token loop runs five kernels (reference order,
// src/main.mojo:538-613 / src/inference/gemma4_e4b.mojo:459-540):
//   1. QKV   : PLE + RMSNorm prologue, fused Q|K|V projection, RoPE, KV write
//   2. attn  : flash-decode GQA over the paged cache
//   3. O     : projection + residual onto the normalised input + row stats
//   4. GU    : RMSNorm prologue, fused gate|up projection, SwiGLU
//   5. Down  : projection + residual + row stats for the next layer's norm
// launched back to back with programmatic dependent launch, so each kernel's
// weight stream starts while its predecessor drains.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types only: the functions are resolved at ms_tp_init (nccl_api)

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/mojostream_cuda.h"
#include "ms_internal.h"
#include "ms_kernels.h"
#include "ms_pages.h"
#include "ms_plan.h"

using namespace ms;

// --------------------------------------------------------------- objects --

struct ms_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  std::string err;
  // scratch shared by the kernels of one stream (consecutive kernels only
  // touch it after griddepcontrol.wait, so one region serves all of them)
  float* part = nullptr;
  size_t part_floats = 0;
  int* counters = nullptr;
  size_t n_counters = 0;
  float* lm_val = nullptr;
  int* lm_idx = nullptr;
  int* lm_counter = nullptr;
  int* d_err = nullptr;  // error bits left by kernels (bounded waits)
  size_t lm_parts = 0;
  // tensor-core projections: activation limb planes and per-row factors
  // (grown on demand outside graph capture; sized up front by ms_model_create)
  uint8_t* lq = nullptr;
  size_t lq_bytes = 0;
  float2* rowf = nullptr;
  size_t rowf_n = 0;
  // ms_sample: chunk partials and per-row arrival tickets (grown on demand)
  float2* samp_part = nullptr;
  size_t samp_part_n = 0;
  double load_secs = 0.0;  // last ms_model_load: reads + host-to-device copies
  uint64_t load_bytes = 0;
  int* samp_cnt = nullptr;
  size_t samp_cnt_n = 0;
  // tensor parallelism (ms_tp_init): heads and FFN columns sharded over ranks
  ncclComm_t comm = nullptr;
  int tp_world = 1, tp_rank = 0;
  cudaEvent_t ev[2] = {nullptr, nullptr};
};

struct LayerDev {
  ms_layer_desc d{};
  int q_dim = 0, kv_dim = 0, qkv_tiles = 0;
  uint4* wqkv = nullptr;
  QkvTile* tiles = nullptr;
  uint4* wo = nullptr;
  uint4* wgu = nullptr;
  uint4* wd = nullptr;
  float* inv_freq = nullptr;
};

struct ms_model {
  ms_ctx* ctx = nullptr;
  unsigned long long uid = 0;  // never reused: a new model may get a freed one's address
  int hidden = 0, n_layers = 0, vocab = 0, max_rows = 0;
  int vocab_local = 0, vocab0 = 0;  // this rank's lm_head columns (all of them without TP)
  float* P = nullptr;               // TP: partial sums of the row-parallel projections
  // TP, tensor-core path: the O / down output tiles are summed over the ranks
  // inside the projection's epilogue through peer memory (CUDA IPC)
  float* sym = nullptr;             // [2][tiles][128 x 128] floats + [2][tiles] use counters
  size_t sym_tiles = 0;
  std::vector<void*> peer_maps;     // other ranks' sym, mapped here
  float** d_peer_tiles = nullptr;   // [2][W] device arrays of pointers
  int** d_peer_flags = nullptr;
  int* d_lidx = nullptr;            // TP: local argmax, its value and the packed keys
  float* d_maxv = nullptr;
  unsigned long long* d_key = nullptr;
  std::vector<LayerDev> layers;
  float* lm_head = nullptr;
  float* gamma = nullptr;
  float* bos = nullptr;  // a loaded lm_head file's BOS embedding (token bos_id)
  int bos_id = -1;
  size_t weight_bytes = 0;
  int max_q = 0, max_f = 0;
  // run buffers (max_rows rows)
  float* X[2] = {nullptr, nullptr};
  float* S[2] = {nullptr, nullptr};
  float* Q = nullptr;
  float* ATT = nullptr;
  float* H = nullptr;
  uint8_t* lq = nullptr;    // tensor-core scratch: limb planes (max_rows x widest K)
  size_t lq_bytes = 0;
  // tensor map over the lm_head table (the tensor-core lm_head), made on first use
  alignas(64) unsigned char lm_map[128];
  int lm_map_state = 0;  // 0 not tried, 1 made, -1 unavailable
  float2* rowf = nullptr;   // and per-row factors
  // prefill attention: query blocks (runs of consecutive positions of one
  // sequence, at most `bq` rows each) of the rows last uploaded, per distinct
  // bq among the layers
  struct QBlocks {
    int bq = 0, n = 0;
    int4* d = nullptr;
  };
  std::vector<QBlocks> qblocks;
  int* d_seq = nullptr;
  int* d_pos = nullptr;
  int* d_ids = nullptr;
  int* d_next = nullptr;
  int* d_step = nullptr;
  int* d_hist = nullptr;
  int hist_cap = 0;
  int* h_stage = nullptr;  // pinned: ids | seq | pos | next (max_rows each) | error word
  // token-loop sampling (ms_set_sampling): greedy without penalty when off
  float samp_t = 0.f, samp_pen = 1.f;
  unsigned long long samp_seed = 0;
  int samp_ver = 0;
  float* d_logits = nullptr;    // [logits_rows][vocab_local], read by the sampler
  int logits_rows = 0;
  float2* d_spart = nullptr;    // [max_rows][chunks] sampler partials
  int* d_scnt = nullptr;        // [max_rows] sampler tickets
  float2* d_rowsum = nullptr;   // TP: this rank's (max, sum) per row
  float2* d_rowsum_all = nullptr;  // TP: [W][max_rows]
  bool sampling() const { return samp_t > 0.01f || samp_pen > 1.f; }
  // captured decode step
  cudaGraphExec_t gexec = nullptr;
  int g_M = 0, g_samp = -1;
  const ms_kv* g_kv = nullptr;
  unsigned long long g_kv_uid = 0;  // the cache's id: a new cache may reuse a freed one's address
  std::vector<void*> allocs;
};

struct ms_kv {
  const ms_model* model = nullptr;
  unsigned long long model_uid = 0;  // the model's uid when the cache was made
  unsigned long long uid = 0;  // never reused (kv_create numbers every cache)
  int n_seq = 0, max_pos = 0, slide_cap = 0, page = 16;
  int pages_full = 0, pages_slide = 0;  // per sequence
  std::vector<float*> k, v;
  int* bt_full = nullptr;
  int* bt_slide = nullptr;
  int* tok = nullptr;  // [n_seq][max_pos] token fed at each position (-1: none)
  int bf16 = 0;        // K / V pools hold bfloat16
  int allow_overwrite = 0;  // calls may overwrite sliding slots still in a window
  // int8 pools (value = int8 * scale, one fp32 scale per position and KV head
  // behind the row's values) and the fp32 rows the projections write before
  // launch_kv_quant moves them in: K [max_rows][stage_ld], then V
  int i8 = 0;
  float* stage = nullptr;
  int stage_ld = 0;
  size_t bytes = 0;
  // pooled mode (ms_kv_create_pooled): the full-attention layers draw pages
  // from one pool of pool_pages pages (a page id indexes every full layer's
  // pool), assigned on first use and shared by reference (prefixes); `pool`
  // is the host side of bt_full with the free list and reference counts
  int pooled = 0, pool_pages = 0;
  PagePool pool;
};

struct ms_q4_weight {
  int K = 0, N = 0;
  float scale = 1.f;
  uint4* w = nullptr;
};

// ----------------------------------------------------------------- errors --

static ms_status fail(ms_ctx* c, ms_status s, const char* fmt, ...) {
  if (c) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    c->err = buf;
  }
  return s;
}

#define MS_CUDA(ctx, call)                                                                   \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return fail((ctx), e_ == cudaErrorMemoryAllocation ? MS_ERR_OOM : MS_ERR_CUDA, "%s: %s", \
                  #call, cudaGetErrorString(e_));                                            \
  } while (0)

#define MS_TRY(expr)               \
  do {                             \
    ms_status s_ = (expr);         \
    if (s_ != MS_OK) return s_;    \
  } while (0)

static cudaStream_t pick(ms_ctx* c, void* s) { return s ? (cudaStream_t)s : c->stream; }

// uint4 words of a fragment-tiled Q4 matrix with K rows and n_tiles tiles
// (padded to whole tile groups).
static size_t q4_u4(int K, int n_tiles) {
  return (size_t)padded_tiles(n_tiles) * kTileN * (size_t)K / 2 / sizeof(uint4);
}

// Fragment rows of buffer X[i] when the call takes the decode path (M <= 8).

// Error bits the kernels leave on the device (a bounded wait that ran out).
// Reading them needs the stream idle; callers use it after a synchronize.
static ms_status check_device_errors(ms_ctx* c) {
  int e = 0;
  if (cudaMemcpy(&e, c->d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(c, MS_ERR_CUDA, "reading the device error word failed");
  if (e) {
    cudaMemset(c->d_err, 0, sizeof(int));
    return fail(c, MS_ERR_TIMEOUT, "a kernel wait ran out (error bits 0x%x)", e);
  }
  return MS_OK;
}

static ms_status dev_alloc(ms_ctx* c, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(c, MS_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  }
  return MS_OK;
}

template <typename T>
static ms_status model_alloc(ms_model* m, T** p, size_t count) {
  void* q = nullptr;
  MS_TRY(dev_alloc(m->ctx, &q, count * sizeof(T)));
  m->allocs.push_back(q);
  *p = (T*)q;
  return MS_OK;
}

static bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// NCCL is resolved on first use instead of linked: a single-GPU host never
// needs it, and in a process that already loaded an NCCL (torch does), the
// same soname resolves to that copy rather than binding it to another one.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

static const NcclApi& nccl_api() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
    a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
    a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
    a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
    a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
    a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
    a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy &&
           a.error_string;
    return a;
  }();
  return api;
}

// ------------------------------------------------------------------ context --

extern "C" int ms_abi_version(void) { return MS_ABI_VERSION; }

extern "C" const char* ms_status_string(ms_status s) {
  switch (s) {
    case MS_OK: return "ok";
    case MS_ERR_INVALID_ARG: return "invalid argument";
    case MS_ERR_SHAPE: return "unsupported shape";
    case MS_ERR_ALIGN: return "misaligned pointer";
    case MS_ERR_CAPACITY: return "capacity exceeded";
    case MS_ERR_CUDA: return "CUDA error";
    case MS_ERR_NCCL: return "NCCL error";
    case MS_ERR_OOM: return "out of device memory";
    case MS_ERR_STATE: return "invalid state";
    case MS_ERR_TIMEOUT: return "timeout";
    case MS_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

extern "C" ms_status ms_init(int device, ms_ctx** out) {
  if (!out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return MS_ERR_CUDA;
  }
  ms_ctx* c = new ms_ctx();
  c->device = device;
  if (cudaSetDevice(device) != cudaSuccess) {
    delete c;
    return MS_ERR_CUDA;
  }
  cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return MS_ERR_CUDA;
  }
  // split-K / attention partials: 32 MiB; tickets: 1 Mi counters
  c->part_floats = (size_t)8 << 20;
  c->n_counters = (size_t)1 << 20;
  c->lm_parts = (size_t)1 << 20;
  if (dev_alloc(c, (void**)&c->part, c->part_floats * sizeof(float)) != MS_OK ||
      dev_alloc(c, (void**)&c->counters, c->n_counters * sizeof(int)) != MS_OK ||
      dev_alloc(c, (void**)&c->lm_val, c->lm_parts * sizeof(float)) != MS_OK ||
      dev_alloc(c, (void**)&c->lm_idx, c->lm_parts * sizeof(int)) != MS_OK ||
      dev_alloc(c, (void**)&c->lm_counter, 64 * sizeof(int)) != MS_OK) {
    ms_destroy(c);
    return MS_ERR_OOM;
  }
  cudaMemset(c->counters, 0, c->n_counters * sizeof(int));
  cudaMemset(c->lm_counter, 0, 64 * sizeof(int));
  if (dev_alloc(c, (void**)&c->d_err, sizeof(int)) != MS_OK) {
    ms_destroy(c);
    return MS_ERR_OOM;
  }
  cudaMemset(c->d_err, 0, sizeof(int));
  cudaEventCreate(&c->ev[0]);
  cudaEventCreate(&c->ev[1]);
  if (prepare_gemv_stream() != cudaSuccess || prepare_attention() != cudaSuccess ||
      prepare_gemm_tc() != cudaSuccess || prepare_gemm_sk() != cudaSuccess ||
      prepare_lm_tc() != cudaSuccess ||
      prepare_attention_prefill() != cudaSuccess) {
    ms_destroy(c);
    return MS_ERR_CUDA;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) {
    ms_destroy(c);
    return MS_ERR_CUDA;
  }
  *out = c;
  return MS_OK;
}

extern "C" ms_status ms_destroy(ms_ctx* c) {
  if (!c) return MS_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  cudaFree(c->part);
  cudaFree(c->counters);
  cudaFree(c->lm_val);
  cudaFree(c->lm_idx);
  cudaFree(c->lm_counter);
  cudaFree(c->d_err);
  cudaFree(c->lq);
  cudaFree(c->rowf);
  cudaFree(c->samp_part);
  cudaFree(c->samp_cnt);
  if (c->comm) nccl_api().comm_destroy(c->comm);
  if (c->ev[0]) cudaEventDestroy(c->ev[0]);
  if (c->ev[1]) cudaEventDestroy(c->ev[1]);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return MS_OK;
}

extern "C" const char* ms_last_error(const ms_ctx* c) { return c ? c->err.c_str() : "null context"; }

// ------------------------------------------------- internal (ms_loader.cu) --

ms_status ms_fail_(ms_ctx* c, ms_status s, const char* msg) { return fail(c, s, "%s", msg); }
cudaStream_t ms_stream_(ms_ctx* c) { return c->stream; }
int ms_device_(const ms_ctx* c) { return c->device; }
void ms_set_load_stats_(ms_ctx* c, double seconds, uint64_t bytes) {
  c->load_secs = seconds;
  c->load_bytes = bytes;
}

extern "C" ms_status ms_load_stats(const ms_ctx* c, double* seconds, uint64_t* bytes) {
  if (!c) return MS_ERR_INVALID_ARG;
  if (seconds) *seconds = c->load_secs;
  if (bytes) *bytes = c->load_bytes;
  return MS_OK;
}

extern "C" ms_status ms_sync(ms_ctx* c, void* stream) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaStreamSynchronize(pick(c, stream)));
  return check_device_errors(c);
}

extern "C" ms_status ms_malloc(ms_ctx* c, size_t bytes, void** dptr) {
  if (!c || !dptr) return MS_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  return dev_alloc(c, dptr, bytes);
}

extern "C" ms_status ms_free(ms_ctx* c, void* dptr) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaFree(dptr));
  return MS_OK;
}

extern "C" ms_status ms_memcpy(ms_ctx* c, void* dst, const void* src, size_t bytes, int kind,
                               void* stream) {
  if (!c || (!dst && bytes) || (!src && bytes)) return MS_ERR_INVALID_ARG;
  cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                               : (kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice);
  if (kind < 0 || kind > 2) return fail(c, MS_ERR_INVALID_ARG, "ms_memcpy: kind %d", kind);
  MS_CUDA(c, cudaMemcpyAsync(dst, src, bytes, k, pick(c, stream)));
  return MS_OK;
}

// ------------------------------------------------------ tensor parallelism --


extern "C" size_t ms_tp_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

extern "C" ms_status ms_tp_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId)) return MS_ERR_INVALID_ARG;
  ncclUniqueId id;
  if (!nccl_api().ok || nccl_api().get_unique_id(&id) != ncclSuccess) return MS_ERR_NCCL;
  memcpy(out, &id, sizeof(id));
  return MS_OK;
}

extern "C" ms_status ms_tp_init(ms_ctx* c, int world, int rank, const void* unique_id) {
  if (!c || !unique_id || world < 1 || rank < 0 || rank >= world) return MS_ERR_INVALID_ARG;
  if (c->comm || c->tp_world > 1) return fail(c, MS_ERR_STATE, "tensor parallelism already set up");
  if (world == 1) return MS_OK;
  MS_CUDA(c, cudaSetDevice(c->device));
  if (!nccl_api().ok) return fail(c, MS_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  const ncclResult_t r = nccl_api().comm_init_rank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    c->comm = nullptr;
    return fail(c, MS_ERR_NCCL, "ncclCommInitRank: %s", nccl_api().error_string(r));
  }
  c->tp_world = world;
  c->tp_rank = rank;
  return MS_OK;
}

extern "C" int ms_tp_world(const ms_ctx* c) { return c ? c->tp_world : 0; }

#define MS_NCCL(c, call)                                                             \
  do {                                                                               \
    const ncclResult_t r_ = (call);                                                  \
    if (r_ != ncclSuccess)                                                           \
      return fail(c, MS_ERR_NCCL, "%s: %s", #call, nccl_api().error_string(r_));    \
  } while (0)

// --------------------------------------------------------- repack helpers --

// Stage a reference-layout matrix on the device (copy if it is host memory).
static ms_status stage_bytes(ms_ctx* c, const uint8_t* src, size_t bytes, const uint8_t** dev,
                             void** owned) {
  *owned = nullptr;
  if (is_device_ptr(src)) {
    *dev = src;
    return MS_OK;
  }
  void* d = nullptr;
  MS_TRY(dev_alloc(c, &d, bytes));
  cudaError_t e = cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return fail(c, MS_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e));
  }
  *dev = (const uint8_t*)d;
  *owned = d;
  return MS_OK;
}

// Repack up to three source matrices (columns concatenated by perm) into
// fragment tiles.
static ms_status repack(ms_ctx* c, uint4* out, const std::vector<const uint8_t*>& srcs,
                        const std::vector<int>& src_n, int K, const std::vector<int>& perm) {
  std::vector<const uint8_t*> dev(srcs.size());
  std::vector<void*> owned(srcs.size(), nullptr);
  ms_status st = MS_OK;
  for (size_t i = 0; i < srcs.size() && st == MS_OK; ++i)
    st = stage_bytes(c, srcs[i], (size_t)K * (src_n[i] / 2), &dev[i], &owned[i]);
  int* dperm = nullptr;
  if (st == MS_OK) st = dev_alloc(c, (void**)&dperm, perm.size() * sizeof(int));
  if (st == MS_OK) {
    cudaMemcpy(dperm, perm.data(), perm.size() * sizeof(int), cudaMemcpyHostToDevice);
    cudaError_t e = launch_repack(out, dev.data(), src_n.data(), (int)srcs.size(), dperm,
                                  (int)perm.size() / kTileN, K, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) st = fail(c, MS_ERR_CUDA, "repack: %s", cudaGetErrorString(e));
  }
  cudaFree(dperm);
  for (void* o : owned) cudaFree(o);
  return st;
}

static std::vector<int> identity_perm(int N, int src = 0) {
  std::vector<int> p(N);
  for (int i = 0; i < N; ++i) p[i] = (src << 24) | i;
  return p;
}

// ----------------------------------------------------------- Q4 weight API --

extern "C" ms_status ms_q4_weight_create(ms_ctx* c, const uint8_t* w_rx, int K, int N,
                                         float scale, ms_q4_weight** out) {
  if (!c || !w_rx || !out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  if (K <= 0 || N <= 0 || K % kChunkK || N % kTileN)
    return fail(c, MS_ERR_SHAPE, "ms_q4_weight_create: K=%d N=%d (need K%%64==0, N%%16==0)", K, N);
  cudaSetDevice(c->device);
  ms_q4_weight* w = new ms_q4_weight();
  w->K = K;
  w->N = N;
  w->scale = scale;
  if (dev_alloc(c, (void**)&w->w, q4_u4(K, N / kTileN) * sizeof(uint4)) != MS_OK) {
    cudaFree(w->w);
    delete w;
    return MS_ERR_OOM;
  }
  ms_status st = repack(c, w->w, {w_rx}, {N}, K, identity_perm(N));
  if (st != MS_OK) {
    cudaFree(w->w);
    delete w;
    return st;
  }
  *out = w;
  return MS_OK;
}

extern "C" ms_status ms_q4_weight_destroy(ms_ctx* c, ms_q4_weight* w) {
  if (!c || !w) return MS_ERR_INVALID_ARG;
  cudaStreamSynchronize(c->stream);
  cudaFree(w->w);
  delete w;
  return MS_OK;
}

// MS_SPLITK_GLOBAL=1: split merges through global memory and arrival tickets
// instead of thread-block clusters (the same sums; for comparisons).
static bool splitk_global_forced() {
  static const bool on = [] {
    const char* e = getenv("MS_SPLITK_GLOBAL");
    return e && e[0] == '1';
  }();
  return on;
}

// Tensor parallel: up to this many rows the O / down all-reduce runs inside
// the tensor-core epilogue over peer memory (measured faster at batch 64 on 2
// GPUs); larger calls use one NCCL all-reduce (faster for 2048-row prefills).
constexpr int kTpFusedMaxRows = 256;

// Grow the tensor-core scratch (limb planes, row factors) to M rows x K.
// Synchronises the context's stream when it allocates; never called while a
// graph is being captured (the model sizes it for max_rows up front).
static ms_status ensure_tc_scratch(ms_ctx* c, int M, int K) {
  const size_t need = tc_limb_bytes(M, K);
  const size_t rows = (size_t)tc_rows_pad(M);
  if (need <= c->lq_bytes && rows <= c->rowf_n) return MS_OK;
  cudaStreamSynchronize(c->stream);
  if (need > c->lq_bytes) {
    cudaFree(c->lq);
    c->lq = nullptr;
    c->lq_bytes = 0;
    MS_TRY(dev_alloc(c, (void**)&c->lq, need));
    c->lq_bytes = need;
  }
  if (rows > c->rowf_n) {
    cudaFree(c->rowf);
    c->rowf = nullptr;
    c->rowf_n = 0;
    MS_TRY(dev_alloc(c, (void**)&c->rowf, rows * sizeof(float2)));
    c->rowf_n = rows;
  }
  return MS_OK;
}

// The projection planner (ms_plan.h) over this context's limits.
static GemvPlan plan_gemv(const ms_ctx* c, int M, int K, int n_tiles, bool allow_tc = true,
                          bool allow_sk = true) {
  const PlanLimits lim{c->sm_count, c->part_floats, c->n_counters, sk_rows_max()};
  return ms::plan_gemv(&lim, M, K, n_tiles, allow_tc, allow_sk);
}

static cudaError_t launch_proj(const GemvParams& p, const GemvPlan& pl, cudaStream_t s, bool pdl) {
  if (pl.sk) return launch_gemm_sk(p, s, pdl);
  if (pl.tc) return launch_gemm_tc(p, s, pdl);
  return pl.dec ? launch_gemv_stream(p, pl.mg, s, pdl) : launch_gemv(p, pl.mg, pl.ch, s, pdl);
}

static GemvParams gemv_base(ms_ctx* c, const uint4* w, int n_tiles, int K, int M,
                            const GemvPlan& pl) {
  GemvParams p{};
  p.w = w;
  p.n_tiles = n_tiles;
  p.K = K;
  p.kseg = pl.kseg;
  p.ksplit = pl.ksplit;
  p.M = M;
  p.in_ple = 1.f;
  p.resid_ple = 1.f;
  p.scale = 1.f;
  p.scale2 = 1.f;
  p.part = c->part;
  p.counters = c->counters;
  p.err = c->d_err;
  p.lq = c->lq;
  p.rowf = c->rowf;
  return p;
}

extern "C" ms_status ms_q4_gemm(ms_ctx* c, const ms_q4_weight* w, float* C, const float* A, int M,
                                int accumulate, void* stream) {
  if (!c || !w || !C || !A) return MS_ERR_INVALID_ARG;
  if (M <= 0) return fail(c, MS_ERR_SHAPE, "ms_q4_gemm: M=%d", M);
  if (((uintptr_t)A & 15) || ((uintptr_t)C & 7))
    return fail(c, MS_ERR_ALIGN, "ms_q4_gemm: A must be 16-byte and C 8-byte aligned");
  const int n_tiles = w->N / kTileN;
  GemvPlan pl = plan_gemv(c, M, w->K, n_tiles);
  if (pl.dec && pl.kseg > decode_seg_max(pl.mg) * kChunkK)
    return fail(c, MS_ERR_CAPACITY,
                "ms_q4_gemm: M=%d K=%d N=%d: the k-split the decode kernel needs for this K "
                "would exceed the context's partial-sum scratch (%zu floats)",
                M, w->K, w->N, c->part_floats);
  if (pl.tc) MS_TRY(ensure_tc_scratch(c, M, w->K));
  GemvParams p = gemv_base(c, w->w, n_tiles, w->K, M, pl);
  p.x = A;
  p.ldx = w->K;
  p.in_D = w->K;
  p.epi = accumulate ? kEpiAccum : kEpiStore;
  p.out = C;
  p.ldo = w->N;
  p.scale = w->scale;
  cudaStream_t s = pick(c, stream);
  MS_CUDA(c, launch_proj(p, pl, s, false));
  return MS_OK;
}

// ------------------------------------------------ allocation-free variant --
// ms_q4_gemm_noalloc runs the same projection as ms_q4_gemm (results within
// the projection tests' 2e-5 relative RMSE: rows above 8 take the CUDA-core
// tiled kernel instead of the tensor-core GEMM, and the k-split is lowered
// when the context's plan would not fit), but its scratch (split-K partial
// sums and arrival tickets) lives in one fixed file-scope device array instead
// of the context's buffers.  Some callers cannot let a call allocate device memory
// or share the context's scratch: a serving host that reserved all of HBM for
// KV pages up front, or code on a latency-critical path where an allocation
// (implicitly synchronising) is not allowed.  This entry point allocates
// nothing, on the device or (on success) on the host.
namespace {
constexpr size_t kNaPartFloats = 256 * 1024;  // 1 MiB of partial sums
constexpr size_t kNaCounters = 4096;          // arrival tickets
constexpr size_t kNaCountOff = kNaPartFloats * sizeof(float);
constexpr size_t kNaBytes = kNaCountOff + kNaCounters * sizeof(int);  // 1 MiB + 16 KiB
constexpr int kNaMaxDevices = 64;
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

// Device address of g_noalloc_scratch per device ordinal, resolved on the
// first call made on that device (with the device current).  Host threads
// may make their first calls at the same time: the lookup runs under a mutex
// and the address is published through an atomic.
static std::atomic<unsigned char*> g_noalloc_addr[kNaMaxDevices];
static std::mutex g_noalloc_mu;

// The largest k-split that fits the static scratch, starting from the
// context's plan and going down to the kernel's smallest split (the decode
// kernel holds at most 40 / 20 k-chunks per segment in registers; the tiled
// kernel runs any K unsplit, which needs no scratch).  False when even that
// does not fit.
static bool noalloc_fit(GemvPlan& pl, int M, int K, int n_tiles) {
  const int chunks = K / kChunkK;
  auto fits = [&](const GemvPlan& q) {
    size_t f = 0, t = 0;
    plan_scratch(q, M, n_tiles, &f, &t);
    return f <= kNaPartFloats && t <= kNaCounters;
  };
  for (int ks = pl.ksplit; ks >= 1; --ks) {
    GemvPlan q = pl;
    if (q.dec) {
      const int seg = (chunks + ks - 1) / ks;
      if (seg > decode_seg_max(q.mg)) break;
      q.kseg = seg * kChunkK;
      q.ksplit = (chunks + seg - 1) / seg;
    } else {
      const int rounds = (chunks + q.ch - 1) / q.ch;
      const int per = (rounds + ks - 1) / ks;
      q.kseg = per * q.ch * kChunkK;
      q.ksplit = (K + q.kseg - 1) / q.kseg;
    }
    if (fits(q)) {
      pl = q;
      return true;
    }
  }
  return false;
}

extern "C" ms_status ms_q4_gemm_noalloc(ms_ctx* c, const ms_q4_weight* w, float* C,
                                        const float* A, int M, int accumulate, void* stream) {
  if (!c || !w || !C || !A) return MS_ERR_INVALID_ARG;
  if (M <= 0) return fail(c, MS_ERR_SHAPE, "ms_q4_gemm_noalloc: M=%d", M);
  if (((uintptr_t)A & 15) || ((uintptr_t)C & 7))
    return fail(c, MS_ERR_ALIGN, "ms_q4_gemm_noalloc: A must be 16-byte and C 8-byte aligned");
  if (c->device < 0 || c->device >= kNaMaxDevices)
    return fail(c, MS_ERR_UNSUPPORTED, "ms_q4_gemm_noalloc: device %d", c->device);
  const int n_tiles = w->N / kTileN;
  // the plan ms_q4_gemm uses, minus the tensor-core path (whose limb
  // buffer grows with M x K): rows above 8 take the CUDA-core tiled kernel
  GemvPlan pl = plan_gemv(c, M, w->K, n_tiles, false);
  if (!noalloc_fit(pl, M, w->K, n_tiles)) {
    size_t need_floats = 0, need_tickets = 0;
    plan_scratch(pl, M, n_tiles, &need_floats, &need_tickets);
    return fail(c, MS_ERR_CAPACITY,
                "ms_q4_gemm_noalloc: M=%d K=%d N=%d needs %zu partial floats and %zu tickets "
                "even at its smallest k-split; the static scratch holds %zu and %zu",
                M, w->K, w->N, need_floats, need_tickets, kNaPartFloats, kNaCounters);
  }
  size_t need_floats = 0, need_tickets = 0;
  plan_scratch(pl, M, n_tiles, &need_floats, &need_tickets);
  MS_CUDA(c, cudaSetDevice(c->device));
  unsigned char* base = g_noalloc_addr[c->device].load(std::memory_order_acquire);
  if (!base) {
    // one-time set-up for this device: look up the array's device address
    // (may load the module, so the first call belongs before any capture)
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    base = g_noalloc_addr[c->device].load(std::memory_order_relaxed);
    if (!base) {
      void* ptr = nullptr;
      MS_CUDA(c, cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
      base = static_cast<unsigned char*>(ptr);
      g_noalloc_addr[c->device].store(base, std::memory_order_release);
    }
  }
  GemvParams p = gemv_base(c, w->w, n_tiles, w->K, M, pl);
  p.part = reinterpret_cast<float*>(base);
  p.counters = reinterpret_cast<int*>(base + kNaCountOff);  // d_err: the context's (ms_sync)
  p.x = A;
  p.ldx = w->K;
  p.in_D = w->K;
  p.epi = accumulate ? kEpiAccum : kEpiStore;
  p.out = C;
  p.ldo = w->N;
  p.scale = w->scale;
  cudaStream_t s = pick(c, stream);
  // tickets must be zero when the kernel starts; a completed launch leaves
  // them zero, and clearing them here also covers a call that timed out
  if (need_tickets) MS_CUDA(c, cudaMemsetAsync(p.counters, 0, need_tickets * sizeof(int), s));
  MS_CUDA(c, launch_proj(p, pl, s, false));
  return MS_OK;
}

// ------------------------------------------------------------------- model --

static ms_status check_layer(ms_ctx* c, const ms_layer_desc& L, int D, int i) {
  if (L.head_dim <= 0 || L.n_heads <= 0 || L.n_kv_heads <= 0 || L.ffn_dim <= 0)
    return fail(c, MS_ERR_SHAPE, "layer %d: non-positive dimension", i);
  if (L.n_heads % L.n_kv_heads)
    return fail(c, MS_ERR_SHAPE, "layer %d: n_heads %% n_kv_heads != 0", i);
  const int G = L.n_heads / L.n_kv_heads;
  const bool hd_ok = L.head_dim == 64 || L.head_dim == 128 || L.head_dim == 256 || L.head_dim == 512;
  const bool g_ok = G == 1 || G == 2 || G == 4 || G == 5 || G == 8;
  if (!hd_ok || !g_ok || (L.head_dim == 512 && G > 4))
    return fail(c, MS_ERR_SHAPE, "layer %d: head_dim %d with %d query heads per KV head not built",
                i, L.head_dim, G);
  if (L.rotary_dims < 0 || L.rotary_dims > L.head_dim || L.rotary_dims % 16 ||
      (L.head_dim - L.rotary_dims) % 16)
    return fail(c, MS_ERR_SHAPE, "layer %d: rotary_dims %d", i, L.rotary_dims);
  if (L.window < 0) return fail(c, MS_ERR_SHAPE, "layer %d: window %d", i, L.window);
  const int q = L.n_heads * L.head_dim, kv = L.n_kv_heads * L.head_dim;
  if (q % kChunkK || L.ffn_dim % kChunkK || kv % kTileN)
    return fail(c, MS_ERR_SHAPE, "layer %d: q_dim %d / ffn %d must be multiples of 64", i, q,
                L.ffn_dim);
  for (int m = 0; m < 7; ++m)
    if (!L.w[m]) return fail(c, MS_ERR_INVALID_ARG, "layer %d: weight %d is null", i, m);
  (void)D;
  return MS_OK;
}

// Column order of the fused Q|K|V matrix: per head, RoPE pairs (i, i + R/2)
// in tiles of 8 + 8, then the unrotated tail in tiles of 16; V plain.
// Tiles of the fused Q|K|V matrix of the local heads (L: the local view);
// source columns are those of heads q_head0.. / kv_head0.. of the full
// matrices, destination columns are local.
static void qkv_layout(const ms_layer_desc& L, std::vector<int>& perm, std::vector<QkvTile>& tiles,
                       int q_head0 = 0, int kv_head0 = 0) {
  const int hd = L.head_dim, R = L.rotary_dims, half = R / 2;
  auto heads = [&](int src, int nh, bool rope) {
    const int sh = (src == 0 ? q_head0 : kv_head0) * hd;  // source column shift
    for (int h = 0; h < nh; ++h) {
      const int base = h * hd;
      int start = 0;
      if (rope) {
        for (int i0 = 0; i0 < half; i0 += 8) {
          QkvTile t{src, base + i0, base + half + i0, i0};
          tiles.push_back(t);
          for (int r = 0; r < 8; ++r) perm.push_back((src << 24) | (sh + base + i0 + r));
          for (int r = 0; r < 8; ++r) perm.push_back((src << 24) | (sh + base + half + i0 + r));
        }
        start = R;
      }
      for (int c0 = start; c0 < hd; c0 += 16) {
        QkvTile t{src, base + c0, base + c0 + 8, -1};
        tiles.push_back(t);
        for (int r = 0; r < 16; ++r) perm.push_back((src << 24) | (sh + base + c0 + r));
      }
    }
  };
  heads(0, L.n_heads, R > 0);
  heads(1, L.n_kv_heads, R > 0);
  heads(2, L.n_kv_heads, false);
}

// Peer-visible tile buffers for the fused all-reduce of the tensor-core O /
// down projections: one allocation per rank (2 buffers of tiles x 128 x 128
// floats + 2 x tiles use counters, zeroed), its IPC handle all-gathered over
// NCCL, the other ranks' allocations mapped into this process.
static ms_status tp_map_peers(ms_ctx* c, ms_model* m, int R, int D) {
  const int W = c->tp_world;
  m->sym_tiles = (size_t)((R + 127) / 128) * ((D + 127) / 128);
  const size_t tile_f = (size_t)128 * 128;
  const size_t bytes = 2 * m->sym_tiles * tile_f * sizeof(float) + 2 * m->sym_tiles * sizeof(int);
  MS_TRY(model_alloc(m, (uint8_t**)&m->sym, bytes));
  MS_CUDA(c, cudaMemset(m->sym, 0, bytes));
  cudaIpcMemHandle_t mine;
  MS_CUDA(c, cudaIpcGetMemHandle(&mine, m->sym));
  cudaIpcMemHandle_t* dh = nullptr;
  MS_TRY(dev_alloc(c, (void**)&dh, W * sizeof(cudaIpcMemHandle_t)));
  ms_status st = MS_OK;
  std::vector<cudaIpcMemHandle_t> all(W);
  if (cudaMemcpy(dh + c->tp_rank, &mine, sizeof(mine), cudaMemcpyHostToDevice) != cudaSuccess)
    st = fail(c, MS_ERR_CUDA, "tp: handle upload");
  if (st == MS_OK) {
    const ncclResult_t r = nccl_api().all_gather(dh + c->tp_rank, dh, sizeof(mine), ncclUint8,
                                                 c->comm, c->stream);
    if (r != ncclSuccess) st = fail(c, MS_ERR_NCCL, "tp handles: %s", nccl_api().error_string(r));
  }
  if (st == MS_OK && (cudaStreamSynchronize(c->stream) != cudaSuccess ||
                      cudaMemcpy(all.data(), dh, W * sizeof(mine), cudaMemcpyDeviceToHost) != cudaSuccess))
    st = fail(c, MS_ERR_CUDA, "tp: handle exchange");
  cudaFree(dh);
  if (st != MS_OK) return st;
  std::vector<float*> tiles(2 * W);
  std::vector<int*> flags(2 * W);
  for (int r = 0; r < W; ++r) {
    uint8_t* base = reinterpret_cast<uint8_t*>(m->sym);
    if (r != c->tp_rank) {
      void* p = nullptr;
      MS_CUDA(c, cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
      m->peer_maps.push_back(p);
      base = static_cast<uint8_t*>(p);
    }
    float* t = reinterpret_cast<float*>(base);
    int* f = reinterpret_cast<int*>(t + 2 * m->sym_tiles * tile_f);
    tiles[r] = t;                                  // O buffer
    tiles[W + r] = t + m->sym_tiles * tile_f;      // down buffer
    flags[r] = f;
    flags[W + r] = f + m->sym_tiles;
  }
  MS_TRY(model_alloc(m, &m->d_peer_tiles, (size_t)2 * W));
  MS_TRY(model_alloc(m, &m->d_peer_flags, (size_t)2 * W));
  MS_CUDA(c, cudaMemcpy(m->d_peer_tiles, tiles.data(), 2 * W * sizeof(float*), cudaMemcpyHostToDevice));
  MS_CUDA(c, cudaMemcpy(m->d_peer_flags, flags.data(), 2 * W * sizeof(int*), cudaMemcpyHostToDevice));
  return MS_OK;
}

extern "C" ms_status ms_model_create(ms_ctx* c, const ms_model_desc* desc, ms_model** out) {
  if (!c || !desc || !out || !desc->layers) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  const int D = desc->hidden;
  if (D <= 0 || D % kChunkK || desc->n_layers <= 0 || desc->max_rows <= 0)
    return fail(c, MS_ERR_SHAPE, "model: hidden %d (multiple of 64), n_layers %d, max_rows %d", D,
                desc->n_layers, desc->max_rows);
  if (desc->vocab < 0 || (desc->vocab > 0 && (!desc->lm_head || desc->vocab % 4)))
    return fail(c, MS_ERR_SHAPE, "model: vocab %d needs an lm_head and vocab %% 4 == 0",
                desc->vocab);
  for (int i = 0; i < desc->n_layers; ++i) MS_TRY(check_layer(c, desc->layers[i], D, i));
  // tensor parallelism: every layer's heads and FFN columns split evenly,
  // local widths on whole 64-k chunks, the vocabulary split evenly
  const int TW = c->tp_world, TR = c->tp_rank;
  for (int i = 0; i < desc->n_layers && TW > 1; ++i) {
    const ms_layer_desc& L = desc->layers[i];
    if (L.n_heads % TW || L.n_kv_heads % TW || L.ffn_dim % (kChunkK * TW) ||
        (L.n_heads / TW * L.head_dim) % kChunkK)
      return fail(c, MS_ERR_SHAPE,
                  "layer %d: %d q heads, %d kv heads, ffn %d do not split over %d ranks", i,
                  L.n_heads, L.n_kv_heads, L.ffn_dim, TW);
  }
  if (TW > 1 && desc->vocab > 0 && (desc->vocab % TW || (desc->vocab / TW) % 4))
    return fail(c, MS_ERR_SHAPE, "vocab %d does not split over %d ranks", desc->vocab, TW);
  cudaSetDevice(c->device);

  static std::atomic<unsigned long long> next_model_uid{1};
  ms_model* m = new ms_model();
  m->ctx = c;
  m->uid = next_model_uid.fetch_add(1);
  m->hidden = D;
  m->n_layers = desc->n_layers;
  m->vocab = desc->vocab;
  m->max_rows = desc->max_rows;
  auto bail = [&](ms_status s) {
    ms_model_destroy(c, m);
    return s;
  };
  for (int i = 0; i < desc->n_layers; ++i) {
    const ms_layer_desc& L = desc->layers[i];  // full shapes
    LayerDev ld;
    ld.d = L;  // the local view: this rank's heads and FFN columns
    ld.d.n_heads = L.n_heads / TW;
    ld.d.n_kv_heads = L.n_kv_heads / TW;
    ld.d.ffn_dim = L.ffn_dim / TW;
    for (int j = 0; j < 7; ++j) ld.d.w[j] = nullptr;
    ld.q_dim = ld.d.n_heads * L.head_dim;
    ld.kv_dim = ld.d.n_kv_heads * L.head_dim;
    const int q_full = L.n_heads * L.head_dim, kv_full = L.n_kv_heads * L.head_dim;
    const int F = ld.d.ffn_dim;
    m->max_q = std::max(m->max_q, ld.q_dim);
    m->max_f = std::max(m->max_f, F);
    // fused Q|K|V of the local heads (column slices of the full matrices)
    std::vector<int> perm;
    std::vector<QkvTile> tiles;
    qkv_layout(ld.d, perm, tiles, TR * ld.d.n_heads, TR * ld.d.n_kv_heads);
    ld.qkv_tiles = (int)tiles.size();
    const int nqkv = ld.q_dim + 2 * ld.kv_dim;
    ms_status st = model_alloc(m, &ld.wqkv, q4_u4(D, (int)tiles.size()));
    if (st == MS_OK) st = repack(c, ld.wqkv, {L.w[0], L.w[1], L.w[2]}, {q_full, kv_full, kv_full}, D, perm);
    if (st == MS_OK) st = model_alloc(m, &ld.tiles, tiles.size());
    if (st == MS_OK)
      cudaMemcpy(ld.tiles, tiles.data(), tiles.size() * sizeof(QkvTile), cudaMemcpyHostToDevice);
    // O: the rows of the local heads (a row slice of [q_full][D/2])
    if (st == MS_OK) st = model_alloc(m, &ld.wo, q4_u4(ld.q_dim, D / kTileN));
    if (st == MS_OK)
      st = repack(c, ld.wo, {L.w[3] + (size_t)TR * ld.q_dim * (D / 2)}, {D}, ld.q_dim,
                  identity_perm(D));
    // gate | up of the local FFN columns, interleaved by 8 columns
    if (st == MS_OK) st = model_alloc(m, &ld.wgu, q4_u4(D, 2 * F / kTileN));
    if (st == MS_OK) {
      std::vector<int> gp;
      gp.reserve(2 * F);
      for (int j = 0; j < F / 8; ++j) {
        for (int r = 0; r < 8; ++r) gp.push_back((0 << 24) | (TR * F + 8 * j + r));
        for (int r = 0; r < 8; ++r) gp.push_back((1 << 24) | (TR * F + 8 * j + r));
      }
      st = repack(c, ld.wgu, {L.w[4], L.w[5]}, {L.ffn_dim, L.ffn_dim}, D, gp);
    }
    // Down: the rows of the local FFN columns
    if (st == MS_OK) st = model_alloc(m, &ld.wd, q4_u4(F, D / kTileN));
    if (st == MS_OK)
      st = repack(c, ld.wd, {L.w[6] + (size_t)TR * F * (D / 2)}, {D}, F, identity_perm(D));
    // RoPE inverse frequencies (src/linalg/kernels.mojo:573-575), fp32 as the
    // reference computes them
    if (st == MS_OK && L.rotary_dims > 0) {
      std::vector<float> inv(L.rotary_dims / 2);
      const float ln_base = logf(L.rope_theta);
      for (int j = 0; j < L.rotary_dims / 2; ++j)
        inv[j] = expf(-(float)(2 * j) / (float)L.rotary_dims * ln_base);
      st = model_alloc(m, &ld.inv_freq, inv.size());
      if (st == MS_OK)
        cudaMemcpy(ld.inv_freq, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice);
    }
    if (st != MS_OK) return bail(st);
    m->weight_bytes += (size_t)D * nqkv / 2 + (size_t)ld.q_dim * D / 2 + (size_t)D * F +
                       (size_t)F * D / 2;
    m->layers.push_back(ld);
  }
  m->vocab_local = desc->vocab / TW;
  m->vocab0 = TR * m->vocab_local;
  if (desc->vocab > 0) {
    // this rank's columns v0 .. v0 + V/TW of the [D][V] table
    const size_t n = (size_t)D * m->vocab_local;
    if (model_alloc(m, &m->lm_head, n) != MS_OK) return bail(MS_ERR_OOM);
    if (cudaMemcpy2D(m->lm_head, (size_t)m->vocab_local * sizeof(float), desc->lm_head + m->vocab0,
                     (size_t)desc->vocab * sizeof(float), (size_t)m->vocab_local * sizeof(float), D,
                     cudaMemcpyDefault) != cudaSuccess)
      return bail(fail(c, MS_ERR_CUDA, "lm_head upload failed"));
    m->weight_bytes += n * sizeof(float);
    if (desc->final_gamma) {
      if (model_alloc(m, &m->gamma, D) != MS_OK) return bail(MS_ERR_OOM);
      cudaMemcpy(m->gamma, desc->final_gamma, D * sizeof(float), cudaMemcpyDefault);
    }
  }
  const int R = desc->max_rows;
  ms_status st = MS_OK;
  if (R >= kTcMinRows) {
    // the model's own tensor-core scratch (its captured graphs keep these
    // pointers, so it is never shared with ms_q4_gemm's growable buffer)
    int kmax = std::max(D, m->max_f);
    kmax = std::max(kmax, m->max_q);
    st = model_alloc(m, &m->lq, tc_limb_bytes(R, kmax));
    if (st == MS_OK) m->lq_bytes = tc_limb_bytes(R, kmax);
    if (st == MS_OK) st = model_alloc(m, &m->rowf, (size_t)tc_rows_pad(R));
  }
  for (const LayerDev& ld : m->layers) {
    const int bq = attention_prefill_tokens(ld.d.head_dim, ld.d.n_heads / ld.d.n_kv_heads);
    bool have = bq <= 0;
    for (const auto& q : m->qblocks) have = have || q.bq == bq;
    if (have || st != MS_OK) continue;
    ms_model::QBlocks q;
    q.bq = bq;
    st = model_alloc(m, &q.d, (size_t)R);
    m->qblocks.push_back(q);
  }
  for (int i = 0; i < 2 && st == MS_OK; ++i) {
    st = model_alloc(m, &m->X[i], (size_t)R * D);
    if (st == MS_OK) st = model_alloc(m, &m->S[i], (size_t)R * (D / kTileN));
  }
  if (st == MS_OK) st = model_alloc(m, &m->Q, (size_t)R * m->max_q);
  if (st == MS_OK) st = model_alloc(m, &m->ATT, (size_t)R * m->max_q);
  if (st == MS_OK) st = model_alloc(m, &m->H, (size_t)R * m->max_f);
  if (st == MS_OK) st = model_alloc(m, &m->d_seq, R);
  if (st == MS_OK) st = model_alloc(m, &m->d_pos, R);
  if (st == MS_OK) st = model_alloc(m, &m->d_ids, R);
  if (st == MS_OK) st = model_alloc(m, &m->d_next, R);
  if (st == MS_OK) st = model_alloc(m, &m->d_step, 1);
  if (st == MS_OK && TW > 1) {
    st = model_alloc(m, &m->P, (size_t)R * D);
    if (st == MS_OK) st = model_alloc(m, &m->d_lidx, R);
    if (st == MS_OK) st = model_alloc(m, &m->d_maxv, R);
    if (st == MS_OK) st = model_alloc(m, &m->d_key, R);
    if (st == MS_OK && R >= kTcMinRows) st = tp_map_peers(c, m, R, D);
  }
  if (st == MS_OK && cudaMallocHost((void**)&m->h_stage, (4 * (size_t)R + 1) * sizeof(int)) != cudaSuccess)
    st = fail(c, MS_ERR_OOM, "pinned staging");
  if (st != MS_OK) return bail(st);
  if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(c, MS_ERR_CUDA, "model upload"));
  *out = m;
  return MS_OK;
}

extern "C" ms_status ms_model_destroy(ms_ctx* c, ms_model* m) {
  if (!c || !m) return MS_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  if (m->gexec) cudaGraphExecDestroy(m->gexec);
  for (void* p : m->peer_maps) cudaIpcCloseMemHandle(p);
  for (void* p : m->allocs) cudaFree(p);
  if (m->d_hist) cudaFree(m->d_hist);
  if (m->d_logits) cudaFree(m->d_logits);
  if (m->h_stage) cudaFreeHost(m->h_stage);
  delete m;
  return MS_OK;
}

extern "C" size_t ms_model_weight_bytes(const ms_model* m) { return m ? m->weight_bytes : 0; }

ms_status ms_model_set_bos_(ms_ctx* c, ms_model* m, const float* bos, int bos_id) {
  if (!m->bos) MS_TRY(model_alloc(m, &m->bos, (size_t)m->hidden));
  MS_CUDA(c, cudaMemcpy(m->bos, bos, m->hidden * sizeof(float), cudaMemcpyDefault));
  m->bos_id = bos_id;
  if (m->gexec) {  // a captured decode step holds the embedding's arguments
    cudaGraphExecDestroy(m->gexec);
    m->gexec = nullptr;
  }
  return MS_OK;
}

// ---------------------------------------------------------------- KV cache --

extern "C" ms_status ms_kv_create(ms_ctx* c, const ms_model* m, int n_seq, int max_pos,
                                  int slide_cap, ms_kv** out) {
  return ms_kv_create_typed(c, m, n_seq, max_pos, slide_cap, MS_KV_F32, out);
}

// Bytes of one cached position of layer L (one of the K or V pools): kv_dim
// values, or for int8 kv_dim bytes then n_kv fp32 scales, padded to 16 bytes.
static size_t kv_row_bytes(const ms_kv* kv, const LayerDev& L) {
  if (kv->i8) return (size_t)L.kv_dim + 16 * (size_t)((L.d.n_kv_heads + 3) / 4);
  return (size_t)L.kv_dim * (kv->bf16 ? 2 : 4);
}
// Pages in layer L's pool, and the pool's bytes (K or V).
static size_t kv_pool_pages(const ms_kv* kv, const LayerDev& L) {
  if (L.d.window == 0 && kv->pooled) return (size_t)kv->pool_pages;
  return (size_t)kv->n_seq * (L.d.window > 0 ? kv->pages_slide : kv->pages_full);
}
static size_t kv_pool_bytes(const ms_kv* kv, const LayerDev& L) {
  return kv_pool_pages(kv, L) * kv->page * kv_row_bytes(kv, L);
}

static ms_status kv_create(ms_ctx* c, const ms_model* m, int n_seq, int max_pos, int slide_cap,
                           int dtype, int pool_pages, ms_kv** out) {
  if (!c || !m || !out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  if (m->ctx != c) return fail(c, MS_ERR_STATE, "model belongs to another context");
  if (n_seq <= 0 || max_pos <= 0 || slide_cap < 0)
    return fail(c, MS_ERR_SHAPE, "kv: n_seq %d max_pos %d slide_cap %d", n_seq, max_pos, slide_cap);
  if (dtype != MS_KV_F32 && dtype != MS_KV_BF16 && dtype != MS_KV_I8)
    return fail(c, MS_ERR_INVALID_ARG, "kv: dtype %d", dtype);
  if (dtype == MS_KV_BF16)
    for (const LayerDev& L : m->layers)
      if (L.kv_dim % 8)
        return fail(c, MS_ERR_SHAPE, "kv: a bf16 cache needs kv_dim %% 8 == 0 (%d)", L.kv_dim);
  if (dtype == MS_KV_I8)
    for (const LayerDev& L : m->layers)
      if (L.d.head_dim % 16)
        return fail(c, MS_ERR_SHAPE, "kv: an int8 cache needs head_dim %% 16 == 0 (%d)",
                    L.d.head_dim);
  cudaSetDevice(c->device);
  static std::atomic<unsigned long long> next_uid{1};
  ms_kv* kv = new ms_kv();
  kv->uid = next_uid.fetch_add(1);
  kv->model = m;
  kv->model_uid = m->uid;
  kv->bf16 = dtype == MS_KV_BF16;
  kv->i8 = dtype == MS_KV_I8;
  kv->n_seq = n_seq;
  kv->max_pos = max_pos;
  int win = 0;
  for (const LayerDev& L : m->layers) win = std::max(win, L.d.window);
  if (win > 0) {
    int cap = slide_cap ? slide_cap : win;
    if (cap < win) {
      delete kv;
      return fail(c, MS_ERR_SHAPE, "kv: slide_cap %d below the window %d", cap, win);
    }
    if (cap % kv->page) {
      delete kv;
      return fail(c, MS_ERR_SHAPE, "kv: slide_cap %d must be a multiple of %d", cap, kv->page);
    }
    kv->slide_cap = cap;
    kv->pages_slide = cap / kv->page;
  }
  kv->pages_full = (max_pos + kv->page - 1) / kv->page;
  auto cleanup = [&](ms_status s) {
    ms_kv_destroy(c, kv);
    return s;
  };
  if (pool_pages > 0) {
    kv->pooled = 1;
    kv->pool_pages = pool_pages;
    kv->pool.init(n_seq, kv->pages_full, pool_pages, kv->page);
  }
  // block tables: sequence s owns pages [s * P, (s + 1) * P) of every pool,
  // except the full-attention pages of a pooled cache (unassigned: -1)
  std::vector<int> bt((size_t)n_seq * std::max(kv->pages_full, kv->pages_slide));
  for (int pass = 0; pass < 2; ++pass) {
    const int P = pass == 0 ? kv->pages_full : kv->pages_slide;
    if (P == 0) continue;
    for (int s = 0; s < n_seq; ++s)
      for (int j = 0; j < P; ++j) bt[(size_t)s * P + j] = (pass == 0 && kv->pooled) ? -1 : s * P + j;
    int** dst = pass == 0 ? &kv->bt_full : &kv->bt_slide;
    if (dev_alloc(c, (void**)dst, (size_t)n_seq * P * sizeof(int)) != MS_OK) return cleanup(MS_ERR_OOM);
    cudaMemcpy(*dst, bt.data(), (size_t)n_seq * P * sizeof(int), cudaMemcpyHostToDevice);
  }
  for (const LayerDev& L : m->layers) {
    const size_t n = kv_pool_bytes(kv, L);
    float *k = nullptr, *v = nullptr;
    if (dev_alloc(c, (void**)&k, n) != MS_OK) return cleanup(MS_ERR_OOM);
    kv->k.push_back(k);
    if (dev_alloc(c, (void**)&v, n) != MS_OK) return cleanup(MS_ERR_OOM);
    kv->v.push_back(v);
    cudaMemset(k, 0, n);
    cudaMemset(v, 0, n);
    kv->bytes += 2 * n;
  }
  if (kv->i8) {
    for (const LayerDev& L : m->layers) kv->stage_ld = std::max(kv->stage_ld, L.kv_dim);
    if (dev_alloc(c, (void**)&kv->stage, 2 * (size_t)m->max_rows * kv->stage_ld * sizeof(float)) !=
        MS_OK)
      return cleanup(MS_ERR_OOM);
  }
  // the repetition-penalty history of every sequence
  if (dev_alloc(c, (void**)&kv->tok, (size_t)n_seq * max_pos * sizeof(int)) != MS_OK)
    return cleanup(MS_ERR_OOM);
  cudaMemset(kv->tok, 0xFF, (size_t)n_seq * max_pos * sizeof(int));
  if (cudaDeviceSynchronize() != cudaSuccess) return cleanup(fail(c, MS_ERR_CUDA, "kv create"));
  *out = kv;
  return MS_OK;
}

extern "C" ms_status ms_kv_create_typed(ms_ctx* c, const ms_model* m, int n_seq, int max_pos,
                                        int slide_cap, int dtype, ms_kv** out) {
  return kv_create(c, m, n_seq, max_pos, slide_cap, dtype, 0, out);
}

extern "C" ms_status ms_kv_create_pooled(ms_ctx* c, const ms_model* m, int n_seq, int max_pos,
                                         int slide_cap, int dtype, int pool_pages, ms_kv** out) {
  if (!c || !out) return MS_ERR_INVALID_ARG;
  if (pool_pages <= 0) return fail(c, MS_ERR_SHAPE, "kv: pool_pages %d", pool_pages);
  return kv_create(c, m, n_seq, max_pos, slide_cap, dtype, pool_pages, out);
}

extern "C" ms_status ms_kv_destroy(ms_ctx* c, ms_kv* kv) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (float* p : kv->k) cudaFree(p);
  for (float* p : kv->v) cudaFree(p);
  cudaFree(kv->bt_full);
  cudaFree(kv->bt_slide);
  cudaFree(kv->tok);
  cudaFree(kv->stage);
  delete kv;
  return MS_OK;
}

extern "C" ms_status ms_kv_reset(ms_ctx* c, ms_kv* kv) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  // positions are explicit per call; the contents need no clearing, but do it
  // so a reset cache is indistinguishable from a new one (a pooled cache
  // also gets all its pages back)
  for (size_t i = 0; i < kv->k.size(); ++i) {
    const size_t n = kv_pool_bytes(kv, kv->model->layers[i]);
    MS_CUDA(c, cudaMemsetAsync(kv->k[i], 0, n, c->stream));
    MS_CUDA(c, cudaMemsetAsync(kv->v[i], 0, n, c->stream));
  }
  MS_CUDA(c, cudaMemsetAsync(kv->tok, 0xFF, (size_t)kv->n_seq * kv->max_pos * sizeof(int), c->stream));
  if (kv->pooled) {
    kv->pool.reset();
    const std::vector<int>& t = kv->pool.table();
    MS_CUDA(c, cudaMemcpyAsync(kv->bt_full, t.data(), t.size() * sizeof(int),
                               cudaMemcpyHostToDevice, c->stream));
  }
  return MS_OK;
}

// ------------------------------------------------------ pooled KV pages --

static std::vector<int> full_layers(const ms_kv* kv) {
  std::vector<int> f;
  for (size_t l = 0; l < kv->model->layers.size(); ++l)
    if (kv->model->layers[l].d.window == 0) f.push_back((int)l);
  return f;
}

// Copy page `from` to page `to` in every full-attention layer's K and V pool.
static ms_status kv_copy_page(ms_ctx* c, ms_kv* kv, int from, int to, cudaStream_t s) {
  for (int l : full_layers(kv)) {
    const size_t row = (size_t)kv->page * kv_row_bytes(kv, kv->model->layers[l]);
    char* k = reinterpret_cast<char*>(kv->k[l]);
    char* v = reinterpret_cast<char*>(kv->v[l]);
    MS_CUDA(c, cudaMemcpyAsync(k + to * row, k + from * row, row, cudaMemcpyDeviceToDevice, s));
    MS_CUDA(c, cudaMemcpyAsync(v + to * row, v + from * row, row, cudaMemcpyDeviceToDevice, s));
  }
  return MS_OK;
}

static ms_status kv_upload_row(ms_ctx* c, ms_kv* kv, int seq, cudaStream_t s) {
  const size_t P = (size_t)kv->pages_full;
  MS_CUDA(c, cudaMemcpyAsync(kv->bt_full + seq * P, kv->pool.row(seq), P * sizeof(int),
                             cudaMemcpyHostToDevice, s));
  return MS_OK;
}

// Pooled cache, before a call that writes positions lo[q] .. hi[q] of each
// sequence q with hi[q] >= 0: assign the pages they need (PagePool::assign),
// then copy the shared pages being replaced and upload the changed rows.
// All or nothing: when the pool runs out, every change of the call is undone
// and nothing is issued on the device.
static ms_status kv_assign_all(ms_ctx* c, ms_kv* kv, const std::vector<int>& lo,
                               const std::vector<int>& hi, cudaStream_t s) {
  PagePool& pool = kv->pool;
  pool.begin();
  std::vector<int> dirty_seqs;
  for (int q = 0; q < (int)hi.size(); ++q) {
    if (hi[q] < 0) continue;
    bool dirty = false;
    const int short_at = pool.assign(q, lo[q], hi[q], &dirty);
    if (short_at >= 0) {
      pool.rollback();
      return fail(c, MS_ERR_CAPACITY,
                  "kv: the page pool (%d pages of %d positions) is exhausted (sequence %d, "
                  "position %d); release finished sequences", kv->pool_pages, kv->page, q,
                  short_at);
    }
    if (dirty) dirty_seqs.push_back(q);
  }
  for (const PagePool::Copy& cp : pool.copies()) MS_TRY(kv_copy_page(c, kv, cp.from, cp.to, s));
  for (int q : dirty_seqs) MS_TRY(kv_upload_row(c, kv, q, s));
  pool.begin();
  return MS_OK;
}

// Before a call that writes rows (seq[r], pos[r]) (and, for a decode loop,
// the `extra` positions after each): assign the pages they need.
static ms_status kv_prepare(ms_ctx* c, ms_kv* kv, const int* seq, const int* pos, int M, int extra,
                            cudaStream_t s) {
  if (!kv->pooled) return MS_OK;
  std::vector<int> lo(kv->n_seq, 1 << 30), hi(kv->n_seq, -1);
  for (int r = 0; r < M; ++r) {
    lo[seq[r]] = std::min(lo[seq[r]], pos[r]);
    hi[seq[r]] = std::max(hi[seq[r]], pos[r] + extra);
  }
  for (int q = 0; q < kv->n_seq; ++q)
    if (hi[q] >= kv->max_pos)
      return fail(c, MS_ERR_CAPACITY, "sequence %d: position %d outside the cache (max_pos %d)", q,
                  hi[q], kv->max_pos);
  return kv_assign_all(c, kv, lo, hi, s);
}

extern "C" ms_status ms_kv_release(ms_ctx* c, ms_kv* kv, int seq) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  if (seq < 0 || seq >= kv->n_seq)
    return fail(c, MS_ERR_INVALID_ARG, "ms_kv_release: sequence %d outside 0..%d", seq,
                kv->n_seq - 1);
  cudaStream_t s = c->stream;
  MS_CUDA(c, cudaMemsetAsync(kv->tok + (size_t)seq * kv->max_pos, 0xFF, kv->max_pos * sizeof(int), s));
  if (!kv->pooled) return MS_OK;
  kv->pool.release(seq);
  return kv_upload_row(c, kv, seq, s);
}

extern "C" ms_status ms_kv_share_prefix(ms_ctx* c, ms_kv* kv, int src, int dst, int n_pos) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  if (src < 0 || src >= kv->n_seq || dst < 0 || dst >= kv->n_seq || src == dst)
    return fail(c, MS_ERR_INVALID_ARG, "ms_kv_share_prefix: sequences %d -> %d", src, dst);
  if (n_pos <= 0 || n_pos > kv->max_pos)
    return fail(c, MS_ERR_CAPACITY, "ms_kv_share_prefix: %d positions (max_pos %d)", n_pos,
                kv->max_pos);
  cudaStream_t s = c->stream;
  const size_t P = (size_t)kv->pages_full;
  if (kv->pooled) {
    // whole pages shared by reference, the page the prefix ends in copied
    PagePool::Copy cp{};
    bool has_copy = false;
    switch (kv->pool.share_prefix(src, dst, n_pos, &cp, &has_copy)) {
      case 0: break;
      case 1:
        return fail(c, MS_ERR_STATE, "ms_kv_share_prefix: sequence %d holds pages (release it)", dst);
      case 2:
        return fail(c, MS_ERR_STATE, "ms_kv_share_prefix: sequence %d lacks a page below position %d",
                    src, n_pos);
      default:
        return fail(c, MS_ERR_CAPACITY, "ms_kv_share_prefix: the page pool is exhausted");
    }
    if (has_copy) MS_TRY(kv_copy_page(c, kv, cp.from, cp.to, s));
    MS_TRY(kv_upload_row(c, kv, dst, s));
  } else {
    // fixed pages: copy the prefix rows of every full-attention layer
    for (int l : full_layers(kv)) {
      const size_t rb = kv_row_bytes(kv, kv->model->layers[l]);
      const size_t bytes = (size_t)n_pos * rb;
      const size_t off = (size_t)P * kv->page * rb;
      char* k = reinterpret_cast<char*>(kv->k[l]);
      char* v = reinterpret_cast<char*>(kv->v[l]);
      MS_CUDA(c, cudaMemcpyAsync(k + dst * off, k + src * off, bytes, cudaMemcpyDeviceToDevice, s));
      MS_CUDA(c, cudaMemcpyAsync(v + dst * off, v + src * off, bytes, cudaMemcpyDeviceToDevice, s));
    }
  }
  // sliding layers: the ring holds position p at slot p % slide_cap in both
  // sequences, so the whole ring is copied (slots past the prefix are
  // overwritten before they are read)
  for (size_t l = 0; l < kv->k.size(); ++l) {
    const LayerDev& L = kv->model->layers[l];
    if (L.d.window == 0) continue;
    const size_t ring = (size_t)kv->pages_slide * kv->page * kv_row_bytes(kv, L);
    char* k = reinterpret_cast<char*>(kv->k[l]);
    char* v = reinterpret_cast<char*>(kv->v[l]);
    MS_CUDA(c, cudaMemcpyAsync(k + dst * ring, k + src * ring, ring, cudaMemcpyDeviceToDevice, s));
    MS_CUDA(c, cudaMemcpyAsync(v + dst * ring, v + src * ring, ring, cudaMemcpyDeviceToDevice, s));
  }
  // the repetition-penalty history of the prefix
  MS_CUDA(c, cudaMemsetAsync(kv->tok + (size_t)dst * kv->max_pos, 0xFF, kv->max_pos * sizeof(int), s));
  MS_CUDA(c, cudaMemcpyAsync(kv->tok + (size_t)dst * kv->max_pos, kv->tok + (size_t)src * kv->max_pos,
                             n_pos * sizeof(int), cudaMemcpyDeviceToDevice, s));
  return MS_OK;
}

extern "C" ms_status ms_kv_allow_window_overwrite(ms_ctx* c, ms_kv* kv, int allow) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  kv->allow_overwrite = allow != 0;
  return MS_OK;
}

extern "C" ms_status ms_kv_pages(const ms_kv* kv, int* used, int* total) {
  if (!kv) return MS_ERR_INVALID_ARG;
  const int tot = kv->pooled ? kv->pool_pages : kv->n_seq * kv->pages_full;
  const int fr = kv->pooled ? kv->pool.free_count() : 0;
  if (used) *used = tot - fr;
  if (total) *total = tot;
  return MS_OK;
}

extern "C" size_t ms_kv_bytes(const ms_kv* kv) { return kv ? kv->bytes : 0; }

static KvView kv_view(const ms_kv* kv, int layer);

// Shared checks of ms_kv_write / ms_kv_read.
static ms_status kv_rows_check(ms_ctx* c, const ms_kv* kv, int layer, int seq, int pos0, int n,
                               const void* k, const void* v, const char* what) {
  if (layer < 0 || layer >= (int)kv->k.size())
    return fail(c, MS_ERR_INVALID_ARG, "%s: layer %d", what, layer);
  if (seq < 0 || seq >= kv->n_seq)
    return fail(c, MS_ERR_INVALID_ARG, "%s: sequence %d outside 0..%d", what, seq, kv->n_seq - 1);
  if (n <= 0 || pos0 < 0 || (long)pos0 + n > kv->max_pos)
    return fail(c, MS_ERR_CAPACITY, "%s: positions %d..%ld outside the cache (max_pos %d)", what,
                pos0, (long)pos0 + n - 1, kv->max_pos);
  if (kv->model->layers[layer].d.window > 0 && n > kv->slide_cap)
    return fail(c, MS_ERR_CAPACITY, "%s: %d positions exceed the sliding ring (%d slots)", what,
                n, kv->slide_cap);
  if (!k || !v) return fail(c, MS_ERR_INVALID_ARG, "%s: null buffer", what);
  if (((uintptr_t)k & 3) || ((uintptr_t)v & 3))
    return fail(c, MS_ERR_ALIGN, "%s: buffers must be 4-byte aligned", what);
  if (kv->i8 && (((uintptr_t)k & 15) || ((uintptr_t)v & 15)))
    return fail(c, MS_ERR_ALIGN, "%s: an int8 cache takes 16-byte aligned buffers", what);
  if (!is_device_ptr(k) || !is_device_ptr(v))
    return fail(c, MS_ERR_INVALID_ARG, "%s: k / v must be device pointers", what);
  return MS_OK;
}

extern "C" ms_status ms_kv_write(ms_ctx* c, ms_kv* kv, int layer, int seq, int pos0, int n,
                                 const float* k, const float* v, void* stream) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  MS_TRY(kv_rows_check(c, kv, layer, seq, pos0, n, k, v, "ms_kv_write"));
  if (kv->pooled && kv->model->layers[layer].d.window == 0) {
    std::vector<int> lo(kv->n_seq, 1 << 30), hi(kv->n_seq, -1);
    lo[seq] = pos0;
    hi[seq] = pos0 + n - 1;
    MS_TRY(kv_assign_all(c, kv, lo, hi, pick(c, stream)));
  }
  MS_CUDA(c, launch_kv_copy(kv_view(kv, layer), seq, pos0, n, const_cast<float*>(k),
                            const_cast<float*>(v), 0, pick(c, stream)));
  return MS_OK;
}

extern "C" ms_status ms_kv_read(ms_ctx* c, const ms_kv* kv, int layer, int seq, int pos0, int n,
                                float* k, float* v, void* stream) {
  if (!c || !kv) return MS_ERR_INVALID_ARG;
  MS_TRY(kv_rows_check(c, kv, layer, seq, pos0, n, k, v, "ms_kv_read"));
  if (kv->pooled && kv->model->layers[layer].d.window == 0)
    for (int j = pos0 / kv->page; j <= (pos0 + n - 1) / kv->page; ++j)
      if (kv->pool.row(seq)[j] < 0)
        return fail(c, MS_ERR_STATE, "ms_kv_read: sequence %d has no page at position %d", seq,
                    j * kv->page);
  MS_CUDA(c, launch_kv_copy(kv_view(kv, layer), seq, pos0, n, k, v, 1, pick(c, stream)));
  return MS_OK;
}

// ----------------------------------------------------------------- forward --

// Host-side validation of one call's rows against the cache.
static ms_status check_rows(ms_ctx* c, const ms_model* m, const ms_kv* kv, const int* seq,
                            const int* pos, int M) {
  if (!seq || !pos) return fail(c, MS_ERR_INVALID_ARG, "seq_ids / pos are null");
  if (M <= 0 || M > m->max_rows)
    return fail(c, MS_ERR_CAPACITY, "M=%d outside 1..max_rows=%d", M, m->max_rows);
  if (kv->model != m || kv->model_uid != m->uid)
    return fail(c, MS_ERR_STATE, "KV cache was made for another model");
  std::set<std::pair<int, int>> seen;
  std::vector<int> pmin(kv->n_seq, 1 << 30), pmax(kv->n_seq, -1);
  for (int r = 0; r < M; ++r) {
    if (seq[r] < 0 || seq[r] >= kv->n_seq)
      return fail(c, MS_ERR_INVALID_ARG, "row %d: sequence %d outside 0..%d", r, seq[r], kv->n_seq - 1);
    if (pos[r] < 0 || pos[r] >= kv->max_pos)
      return fail(c, MS_ERR_CAPACITY, "row %d: position %d outside the cache (max_pos %d)", r,
                  pos[r], kv->max_pos);
    if (!seen.insert({seq[r], pos[r]}).second)
      return fail(c, MS_ERR_INVALID_ARG, "row %d: (sequence %d, position %d) given twice", r,
                  seq[r], pos[r]);
    pmin[seq[r]] = std::min(pmin[seq[r]], pos[r]);
    pmax[seq[r]] = std::max(pmax[seq[r]], pos[r]);
  }
  if (kv->slide_cap > 0 && !kv->allow_overwrite) {
    int win = 0;
    for (const LayerDev& L : m->layers) win = std::max(win, L.d.window);
    for (int s = 0; s < kv->n_seq; ++s)
      if (pmax[s] >= 0 && pmax[s] - pmin[s] + win > kv->slide_cap)
        return fail(c, MS_ERR_CAPACITY,
                    "sequence %d: positions %d..%d in one call overwrite sliding slots still in "
                    "the window (slide_cap %d)", s, pmin[s], pmax[s], kv->slide_cap);
  }
  return MS_OK;
}

static ms_status upload_rows(ms_ctx* c, ms_model* m, const int* seq, const int* pos, int M,
                             cudaStream_t s) {
  MS_CUDA(c, cudaMemcpyAsync(m->d_seq, seq, M * sizeof(int), cudaMemcpyHostToDevice, s));
  MS_CUDA(c, cudaMemcpyAsync(m->d_pos, pos, M * sizeof(int), cudaMemcpyHostToDevice, s));
  // query blocks for the prefill attention kernel: a block continues while the
  // next row is the same sequence at the next position and it has room
  for (auto& q : m->qblocks) {
    std::vector<int4> b;
    for (int r = 0; r < M; ++r) {
      if (!b.empty() && seq[r] == b.back().z && pos[r] == b.back().w + b.back().y &&
          b.back().y < q.bq)
        ++b.back().y;
      else
        b.push_back(make_int4(r, 1, seq[r], pos[r]));
    }
    q.n = (int)b.size();
    // pageable source: the copy has taken the data when the call returns
    MS_CUDA(c, cudaMemcpyAsync(q.d, b.data(), b.size() * sizeof(int4), cudaMemcpyHostToDevice, s));
  }
  return MS_OK;
}

static KvView kv_view(const ms_kv* kv, int layer) {
  const LayerDev& L = kv->model->layers[layer];
  KvView v{};
  v.k = kv->k[layer];
  v.v = kv->v[layer];
  const bool slide = L.d.window > 0;
  v.block_table = slide ? kv->bt_slide : kv->bt_full;
  v.bt_stride = slide ? kv->pages_slide : kv->pages_full;
  v.page = kv->page;
  v.cap = slide ? kv->slide_cap : kv->pages_full * kv->page;
  v.circular = slide ? 1 : 0;
  v.kv_dim = L.kv_dim;
  const size_t pages = (!slide && kv->pooled) ? (size_t)kv->pool_pages
                                              : (size_t)kv->n_seq * v.bt_stride;
  v.off32 = pages * v.page * v.kv_dim < ((size_t)1 << 32);
  v.bf16 = kv->bf16;
  v.i8 = kv->i8;
  v.row_bytes = (int)kv_row_bytes(kv, L);
  v.hd = L.d.head_dim;
  if (kv->i8) {
    v.stage_k = kv->stage;
    v.stage_v = kv->stage + (size_t)kv->model->max_rows * kv->stage_ld;
  }
  return v;
}

// The five kernels of one layer.  x/xs: input rows and their stats (in
// place: the layer output lands in x, its stats in xs); y/ys: the second
// residual buffer.
static ms_status run_layer(ms_ctx* c, ms_model* m, const ms_kv* kv, int li, int M, float* x,
                           float* xs, float* y, float* ys, cudaStream_t s, bool pdl,
                           bool blocks_valid) {
  const LayerDev& L = m->layers[li];
  const int D = m->hidden, F = L.d.ffn_dim, nstat = D / kTileN;
  // 1. QKV + RoPE + KV write
  {
    GemvPlan pl = plan_gemv(c, M, D, L.qkv_tiles);
    GemvParams p = gemv_base(c, L.wqkv, L.qkv_tiles, D, M, pl);
    p.lq = m->lq;
    p.rowf = m->rowf;
    p.x = x;
    p.ldx = D;
    p.in_stats = xs;
    p.in_nstat = nstat;
    p.in_ple = L.d.ple;
    p.in_D = D;
    p.epi = kEpiQKV;
    p.tiles = L.tiles;
    p.sq = L.d.scale[0];
    p.sk = L.d.scale[1];
    p.sv = L.d.scale[2];
    p.q_out = m->Q;
    p.ldq = L.q_dim;
    p.inv_freq = L.inv_freq;
    p.pos = m->d_pos;
    p.seq = m->d_seq;
    p.kv = kv_view(kv, li);
    MS_CUDA(c, launch_proj(p, pl, s, pdl));
    if (kv->i8) MS_CUDA(c, launch_kv_quant(p.kv, m->d_seq, m->d_pos, M, s, pdl));
  }
  // 2. attention
  {
    AttnParams a{};
    a.q = m->Q;
    a.ldq = L.q_dim;
    a.out = m->ATT;
    a.ldo = L.q_dim;
    a.kv = kv_view(kv, li);
    a.seq = m->d_seq;
    a.pos = m->d_pos;
    a.hd = L.d.head_dim;
    a.n_heads = L.d.n_heads;
    a.n_kv = L.d.n_kv_heads;
    a.window = L.d.window;
    a.M = M;
    a.scale = 1.0f / sqrtf((float)L.d.head_dim);
    // position splits and their merge (ms_plan.h) at the longest span the
    // cache can hold, so one launch shape serves every position
    const int span = L.d.window > 0 ? std::min(L.d.window, kv->max_pos) : kv->max_pos;
    const int G = L.d.n_heads / L.d.n_kv_heads;
    const AttnLimits al{c->sm_count, c->part_floats, attention_max_splits(),
                        attention_max_cluster(), splitk_global_forced()};
    const AttnPlan ap = plan_attention(&al, M, L.d.n_kv_heads, G, L.d.head_dim, span);
    a.cluster = ap.cluster;
    if ((size_t)M * L.d.n_kv_heads > c->n_counters)
      return fail(c, MS_ERR_CAPACITY, "attention: too many rows for the ticket counters");
    a.chunk = kAttnMinPerSplit;
    a.n_splits = ap.splits;
    a.part = c->part;
    a.counters = c->counters;
    a.err = c->d_err;
    // prefill chunks (query blocks of 4+ rows on average) take the tiled
    // kernel; decode rows and scattered rows the flash-decode kernel
    const ms_model::QBlocks* qb = nullptr;
    const int bq = attention_prefill_tokens(L.d.head_dim, G);
    if (blocks_valid && M > 8 && bq > 0)
      for (const auto& q : m->qblocks)
        if (q.bq == bq && q.n > 0 && M >= 4 * q.n) qb = &q;
    if (qb) {
      a.blocks = qb->d;
      a.n_blocks = qb->n;
      MS_CUDA(c, launch_attention_prefill(a, s, pdl));
    } else {
      MS_CUDA(c, launch_attention(a, s, pdl));
    }
  }
  // 3. O projection + residual onto the normalised input (tensor parallel:
  //    partial sums, all-reduce, then the residual)
  const bool tp = c->tp_world > 1;
  {
    // tensor parallel: the decode-batch kernel sums the ranks' tiles in its
    // cluster epilogue (so it needs k-slices), the prefill GEMM in its own
    GemvPlan pl = plan_gemv(c, M, L.q_dim, D / kTileN);
    if (tp && pl.sk && pl.ksplit < 2) pl = plan_gemv(c, M, L.q_dim, D / kTileN, true, false);
    GemvParams p = gemv_base(c, L.wo, D / kTileN, L.q_dim, M, pl);
    p.lq = m->lq;
    p.rowf = m->rowf;
    p.x = m->ATT;
    p.ldx = L.q_dim;
    p.in_D = D;
    p.epi = kEpiResid;
    p.out = y;
    p.ldo = D;
    p.scale = L.d.scale[3];
    p.resid = x;
    p.ldr = D;
    p.resid_stats = xs;
    p.resid_nstat = nstat;
    p.resid_ple = L.d.ple;
    p.out_stats = ys;
    // all-reduce inside the epilogue for decode batches; prefill chunks (many
    // row tiles) move their partials with one NCCL all-reduce instead
    const bool fused = tp && pl.tc && m->d_peer_tiles && M <= kTpFusedMaxRows;
    if (fused) {
      p.peer_tiles = m->d_peer_tiles;
      p.peer_flags = m->d_peer_flags;
      p.tp_world = c->tp_world;
      p.tp_rank = c->tp_rank;
    } else if (tp) {
      p.epi = kEpiStore;
      p.out = m->P;
    }
    MS_CUDA(c, launch_proj(p, pl, s, pdl));
    if (tp && !fused) {
      MS_NCCL(c, nccl_api().all_reduce(m->P, m->P, (size_t)M * D, ncclFloat, ncclSum, c->comm, s));
      MS_CUDA(c, launch_resid_add(y, ys, m->P, x, xs, L.d.ple, M, D, s));
    }
  }
  // 4. gate | up + SwiGLU
  {
    const int nt = 2 * F / kTileN;
    GemvPlan pl = plan_gemv(c, M, D, nt);
    GemvParams p = gemv_base(c, L.wgu, nt, D, M, pl);
    p.lq = m->lq;
    p.rowf = m->rowf;
    p.x = y;
    p.ldx = D;
    p.in_stats = ys;
    p.in_nstat = nstat;
    p.in_D = D;
    p.epi = kEpiSwiGLU;
    p.out = m->H;
    p.ldo = F;
    p.scale = L.d.scale[4];
    p.scale2 = L.d.scale[5];
    MS_CUDA(c, launch_proj(p, pl, s, pdl));
  }
  // 5. Down + residual
  {
    GemvPlan pl = plan_gemv(c, M, F, D / kTileN);
    if (tp && pl.sk && pl.ksplit < 2) pl = plan_gemv(c, M, F, D / kTileN, true, false);
    GemvParams p = gemv_base(c, L.wd, D / kTileN, F, M, pl);
    p.lq = m->lq;
    p.rowf = m->rowf;
    p.x = m->H;
    p.ldx = F;
    p.in_D = D;
    p.epi = kEpiResid;
    p.out = x;
    p.ldo = D;
    p.scale = L.d.scale[6];
    p.resid = y;
    p.ldr = D;
    p.resid_stats = ys;
    p.resid_nstat = nstat;
    p.resid_ple = 1.f;
    p.out_stats = xs;
    const bool fused = tp && pl.tc && m->d_peer_tiles && M <= kTpFusedMaxRows;
    if (fused) {
      p.peer_tiles = m->d_peer_tiles + c->tp_world;  // the down buffers
      p.peer_flags = m->d_peer_flags + c->tp_world;
      p.tp_world = c->tp_world;
      p.tp_rank = c->tp_rank;
    } else if (tp) {
      p.epi = kEpiStore;
      p.out = m->P;
    }
    MS_CUDA(c, launch_proj(p, pl, s, pdl));
    if (tp && !fused) {
      MS_NCCL(c, nccl_api().all_reduce(m->P, m->P, (size_t)M * D, ncclFloat, ncclSum, c->comm, s));
      MS_CUDA(c, launch_resid_add(x, xs, m->P, y, ys, 1.f, M, D, s));
    }
  }
  return MS_OK;
}

static ms_status check_x(ms_ctx* c, const float* x) {
  if (!x) return fail(c, MS_ERR_INVALID_ARG, "x is null");
  if ((uintptr_t)x & 15) return fail(c, MS_ERR_ALIGN, "x must be 16-byte aligned");
  return MS_OK;
}

extern "C" ms_status ms_layer_forward(ms_ctx* c, const ms_model* mc, int layer, float* x,
                                      ms_kv* kv, const int* seq, const int* pos, int M,
                                      void* stream) {
  if (!c || !mc || !kv) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  if (layer < 0 || layer >= m->n_layers) return fail(c, MS_ERR_INVALID_ARG, "layer %d", layer);
  MS_TRY(check_x(c, x));
  MS_TRY(check_rows(c, m, kv, seq, pos, M));
  cudaStream_t s = pick(c, stream);
  MS_TRY(kv_prepare(c, kv, seq, pos, M, 0, s));
  MS_TRY(upload_rows(c, m, seq, pos, M, s));
  MS_CUDA(c, launch_rowstats(m->S[0], x, m->hidden, M, m->hidden, s, false));
  return run_layer(c, m, kv, layer, M, x, m->S[0], m->X[1], m->S[1], s, true, true);
}

extern "C" ms_status ms_forward(ms_ctx* c, const ms_model* mc, float* x, ms_kv* kv,
                                const int* seq, const int* pos, int M, void* stream) {
  if (!c || !mc || !kv) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  MS_TRY(check_x(c, x));
  MS_TRY(check_rows(c, m, kv, seq, pos, M));
  cudaStream_t s = pick(c, stream);
  MS_TRY(kv_prepare(c, kv, seq, pos, M, 0, s));
  MS_TRY(upload_rows(c, m, seq, pos, M, s));
  MS_CUDA(c, launch_rowstats(m->S[0], x, m->hidden, M, m->hidden, s, false));
  for (int l = 0; l < m->n_layers; ++l)
    MS_TRY(run_layer(c, m, kv, l, M, x, m->S[0], m->X[1], m->S[1], s, true, true));
  return MS_OK;
}

static ms_status lm_head_launch(ms_ctx* c, ms_model* m, const float* x, const float* stats, int M,
                                float* logits, int* argmax, cudaStream_t s, bool pdl) {
  LmHeadParams p{};
  p.x = x;
  p.stats = stats;
  p.nstat = m->hidden / kTileN;
  p.gamma = m->gamma;
  p.W = m->lm_head;
  p.D = m->hidden;
  p.V = m->vocab_local;  // this rank's columns (all of them without TP)
  p.M = M;
  p.logits = logits;
  p.part_val = c->lm_val;
  p.part_idx = c->lm_idx;
  p.counter = c->lm_counter;
  p.argmax = argmax;
  const bool tp = c->tp_world > 1 && argmax;
  if (tp) {  // local argmax and its value, then the combine over ranks
    p.argmax = m->d_lidx;
    p.maxval = m->d_maxv;
  }
  p.planes = m->lq;
  p.planes_bytes = m->lq_bytes;
  p.err = c->d_err;
  // batches of 9+ rows: the tensor-core kernel (two persistent CTAs per SM,
  // one read of the table per 64 rows); up to 8 rows: the CUDA-core kernel
  // fed by a ring of tensor copies (one persistent CTA per SM), or, when its
  // rows do not fit beside the ring, the register-staged CUDA-core kernel
  bool tc = lm_tc_ok(p), ring = !tc && lm_ring_ok(p);
  if ((tc || ring) && m->lm_map_state == 0)
    m->lm_map_state = lm_tc_make_map(m->lm_map, m->lm_head, m->hidden, m->vocab_local) ? 1 : -1;
  tc = tc && m->lm_map_state == 1;
  ring = ring && m->lm_map_state == 1;
  const size_t ctas = tc ? (size_t)2 * c->sm_count
                          : ring ? (size_t)c->sm_count : (m->vocab_local + 511) / 512;
  if (ctas * M > c->lm_parts) return fail(c, MS_ERR_CAPACITY, "lm_head: too many rows");
  if (tc)
    MS_CUDA(c, launch_lm_tc(p, m->lm_map, (int)ctas, s, pdl));
  else if (ring)
    MS_CUDA(c, launch_lm_ring(p, m->lm_map, (int)ctas, s, pdl));
  else
    MS_CUDA(c, launch_lm_head(p, s, pdl));
  if (tp) {
    MS_CUDA(c, launch_argmax_pack(m->d_key, m->d_maxv, m->d_lidx, M, m->vocab0, s));
    MS_NCCL(c, nccl_api().all_reduce(m->d_key, m->d_key, M, ncclUint64, ncclMax, c->comm, s));
    MS_CUDA(c, launch_argmax_unpack(argmax, m->d_key, M, s));
  }
  return MS_OK;
}

// Buffers of the token-loop sampler; the logits block grows to `rows` rows
// (outside graph capture; a captured decode step holding the old block is
// dropped).
static ms_status ensure_sampler(ms_ctx* c, ms_model* m, int rows) {
  if (!m->d_spart) {
    const size_t nch = (m->vocab_local + kSampChunk - 1) / kSampChunk;
    MS_TRY(model_alloc(m, &m->d_spart, (size_t)m->max_rows * nch));
    MS_TRY(model_alloc(m, &m->d_scnt, (size_t)m->max_rows));
    MS_CUDA(c, cudaMemset(m->d_scnt, 0, m->max_rows * sizeof(int)));
    if (c->tp_world > 1) {
      MS_TRY(model_alloc(m, &m->d_rowsum, (size_t)m->max_rows));
      MS_TRY(model_alloc(m, &m->d_rowsum_all, (size_t)c->tp_world * m->max_rows));
    }
  }
  if (m->logits_rows < rows) {
    MS_CUDA(c, cudaStreamSynchronize(c->stream));
    if (m->gexec) {
      cudaGraphExecDestroy(m->gexec);
      m->gexec = nullptr;
    }
    cudaFree(m->d_logits);
    m->d_logits = nullptr;
    m->logits_rows = 0;
    MS_TRY(dev_alloc(c, (void**)&m->d_logits, (size_t)rows * m->vocab_local * sizeof(float)));
    m->logits_rows = rows;
  }
  return MS_OK;
}

// temperature_sampling (lm_head.mojo:198-254) of the M rows in d_logits into
// out (device ids).  History: the cache's token table up to each row's
// position; seed of a row: splitmix64(seed ^ (seq << 32 | pos)).  Tensor
// parallel: greedy combines (value, index) keys like the plain argmax; with a
// temperature the ranks all-gather their (max, sum) per row and the rank that
// holds the target picks (an all-reduce max leaves its id everywhere).
static ms_status sample_rows(ms_ctx* c, ms_model* m, const ms_kv* kv, int M, const int* seq,
                             const int* pos, int* out, cudaStream_t s) {
  SampleParams p{};
  p.logits = m->d_logits;
  p.ld = m->vocab_local;
  p.M = M;
  p.V = m->vocab_local;
  p.v0 = m->vocab0;
  p.nchunk = (m->vocab_local + kSampChunk - 1) / kSampChunk;
  p.tok = kv ? kv->tok : nullptr;
  p.seq = seq;
  p.pos = pos;
  p.tok_ld = kv ? kv->max_pos : 0;
  p.temperature = m->samp_t;
  p.penalty = m->samp_pen;
  p.seed = m->samp_seed;
  p.part = m->d_spart;
  p.counter = m->d_scnt;
  p.tp_world = c->tp_world;
  p.tp_rank = c->tp_rank;
  if (c->tp_world == 1) {
    p.out = out;
    MS_CUDA(c, launch_sample(p, s));
    return MS_OK;
  }
  if (m->samp_t <= 0.01f) {
    p.out = m->d_lidx;
    p.maxval = m->d_maxv;
    MS_CUDA(c, launch_sample(p, s));
    MS_CUDA(c, launch_argmax_pack(m->d_key, m->d_maxv, m->d_lidx, M, m->vocab0, s));
    MS_NCCL(c, nccl_api().all_reduce(m->d_key, m->d_key, M, ncclUint64, ncclMax, c->comm, s));
    MS_CUDA(c, launch_argmax_unpack(out, m->d_key, M, s));
    return MS_OK;
  }
  p.rowsum = m->d_rowsum;
  MS_CUDA(c, launch_sample(p, s));
  MS_NCCL(c, nccl_api().all_gather(m->d_rowsum, m->d_rowsum_all, 2 * (size_t)M, ncclFloat,
                                   c->comm, s));
  p.rowsum = nullptr;
  p.rowsum_all = m->d_rowsum_all;
  p.out = out;
  MS_CUDA(c, launch_sample_pick(p, s));
  MS_NCCL(c, nccl_api().all_reduce(out, out, M, ncclInt32, ncclMax, c->comm, s));
  return MS_OK;
}

// Embedding rows of d_ids into x (+ stats in S[0]).  Tensor parallel: every
// rank gathers the ids in its vocabulary slice, an all-reduce sums the rows.
// With a cache, the ids are also recorded at (d_seq, d_pos) in its token
// table (the repetition-penalty history).
static ms_status embed_rows(ms_ctx* c, ms_model* m, float* x, int M, cudaStream_t s, bool pdl,
                            const ms_kv* kv = nullptr) {
  const TokenLog log{kv ? kv->tok : nullptr, kv ? kv->max_pos : 0, m->d_seq, m->d_pos};
  MS_CUDA(c, launch_embed_stats(x, m->S[0], m->lm_head, m->d_ids, M, m->hidden, m->vocab_local, s,
                                pdl, m->vocab0, log, m->bos, m->bos_id));
  if (c->tp_world > 1) {
    MS_NCCL(c, nccl_api().all_reduce(x, x, (size_t)M * m->hidden, ncclFloat, ncclSum, c->comm, s));
    MS_CUDA(c, launch_rowstats(m->S[0], x, m->hidden, M, m->hidden, s, false));
  }
  return MS_OK;
}

static ms_status embed_ids(ms_ctx* c, ms_model* m, const int* ids, int M, float* x,
                           cudaStream_t s, const ms_kv* kv) {
  if (m->vocab <= 0) return fail(c, MS_ERR_STATE, "model has no embedding table");
  if (M <= 0 || M > m->max_rows) return fail(c, MS_ERR_CAPACITY, "M=%d", M);
  for (int r = 0; r < M; ++r)
    if (ids[r] < 0 || ids[r] >= m->vocab)
      return fail(c, MS_ERR_INVALID_ARG, "token id %d outside 0..%d", ids[r], m->vocab - 1);
  MS_CUDA(c, cudaMemcpyAsync(m->d_ids, ids, M * sizeof(int), cudaMemcpyHostToDevice, s));
  return embed_rows(c, m, x, M, s, false, kv);
}

extern "C" ms_status ms_embed(ms_ctx* c, const ms_model* mc, const int* ids, int M, float* x,
                              void* stream) {
  if (!c || !mc || !ids) return MS_ERR_INVALID_ARG;
  MS_TRY(check_x(c, x));
  return embed_ids(c, const_cast<ms_model*>(mc), ids, M, x, pick(c, stream), nullptr);
}

extern "C" ms_status ms_lm_head(ms_ctx* c, const ms_model* mc, const float* x, int M,
                                float* logits, int* argmax_out, void* stream) {
  if (!c || !mc) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  MS_TRY(check_x(c, x));
  if (m->vocab <= 0) return fail(c, MS_ERR_STATE, "model has no lm_head");
  if (M <= 0 || M > m->max_rows) return fail(c, MS_ERR_CAPACITY, "M=%d", M);
  if (logits && ((uintptr_t)logits & 15)) return fail(c, MS_ERR_ALIGN, "logits must be 16-byte aligned");
  cudaStream_t s = pick(c, stream);
  MS_CUDA(c, launch_rowstats(m->S[1], x, m->hidden, M, m->hidden, s, false));
  return lm_head_launch(c, m, x, m->S[1], M, logits, argmax_out, s, true);
}

// One decode step on the device: d_ids / d_seq / d_pos -> d_next.
static ms_status decode_body(ms_ctx* c, ms_model* m, const ms_kv* kv, int M, cudaStream_t s) {
  MS_TRY(embed_rows(c, m, m->X[0], M, s, true, kv));
  for (int l = 0; l < m->n_layers; ++l)
    MS_TRY(run_layer(c, m, kv, l, M, m->X[0], m->S[0], m->X[1], m->S[1], s, true, false));
  if (m->sampling()) {
    MS_TRY(lm_head_launch(c, m, m->X[0], m->S[0], M, m->d_logits, nullptr, s, true));
    MS_TRY(sample_rows(c, m, kv, M, m->d_seq, m->d_pos, m->d_next, s));
  } else {
    MS_TRY(lm_head_launch(c, m, m->X[0], m->S[0], M, nullptr, m->d_next, s, true));
  }
  return MS_OK;
}

// The decode step captured as a CUDA graph.  No launch shape depends on the
// positions (they are read from d_pos on the device), so one graph serves a
// whole generation.  The graph holds the cache's device pointers, so it is
// reused only for the same cache: same address and same id (a cache created
// after another was destroyed can get its address).
static ms_status ensure_graph(ms_ctx* c, ms_model* m, const ms_kv* kv, int M) {
  if (m->gexec && m->g_M == M && m->g_kv == kv && m->g_kv_uid == kv->uid &&
      m->g_samp == m->samp_ver)
    return MS_OK;
  if (m->gexec) {
    cudaGraphExecDestroy(m->gexec);
    m->gexec = nullptr;
  }
  if (m->sampling()) MS_TRY(ensure_sampler(c, m, M));
  cudaStream_t s = c->stream;
  cudaGraph_t g = nullptr;
  MS_CUDA(c, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  ms_status st = decode_body(c, m, kv, M, s);
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (st != MS_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (e != cudaSuccess) return fail(c, MS_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&m->gexec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(c, MS_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
  m->g_M = M;
  m->g_kv = kv;
  m->g_kv_uid = kv->uid;
  m->g_samp = m->samp_ver;
  return MS_OK;
}

// Validate a decode call and stage its rows (ids / seq / pos) through pinned
// host memory into the device row buffers.
static ms_status stage_rows(ms_ctx* c, ms_model* m, ms_kv* kv, const int* ids,
                            const int* seq, const int* pos, int M, int steps, cudaStream_t s) {
  if (m->vocab <= 0) return fail(c, MS_ERR_STATE, "model has no lm_head");
  MS_TRY(check_rows(c, m, kv, seq, pos, M));
  if (steps > 1) {  // every position the loop reaches must fit the cache
    std::vector<int> last(pos, pos + M);
    for (int& p : last) p += steps - 1;
    MS_TRY(check_rows(c, m, kv, seq, last.data(), M));
  }
  MS_TRY(kv_prepare(c, kv, seq, pos, M, steps - 1, s));
  for (int r = 0; r < M; ++r)
    if (ids[r] < 0 || ids[r] >= m->vocab)
      return fail(c, MS_ERR_INVALID_ARG, "token id %d outside 0..%d", ids[r], m->vocab - 1);
  int* h = m->h_stage;
  memcpy(h, ids, M * sizeof(int));
  memcpy(h + m->max_rows, seq, M * sizeof(int));
  memcpy(h + 2 * m->max_rows, pos, M * sizeof(int));
  MS_CUDA(c, cudaMemcpyAsync(m->d_ids, h, M * sizeof(int), cudaMemcpyHostToDevice, s));
  MS_CUDA(c, cudaMemcpyAsync(m->d_seq, h + m->max_rows, M * sizeof(int), cudaMemcpyHostToDevice, s));
  MS_CUDA(c, cudaMemcpyAsync(m->d_pos, h + 2 * m->max_rows, M * sizeof(int), cudaMemcpyHostToDevice, s));
  return MS_OK;
}

extern "C" ms_status ms_decode_step(ms_ctx* c, const ms_model* mc, ms_kv* kv, const int* ids,
                                    const int* seq, const int* pos, int M, int* next_ids) {
  if (!c || !mc || !kv || !ids || !next_ids) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  cudaStream_t s = c->stream;
  MS_TRY(stage_rows(c, m, kv, ids, seq, pos, M, 1, s));
  MS_TRY(ensure_graph(c, m, kv, M));
  MS_CUDA(c, cudaGraphLaunch(m->gexec, s));
  int* h_next = m->h_stage + 3 * m->max_rows;
  int* h_err = m->h_stage + 4 * m->max_rows;
  MS_CUDA(c, cudaMemcpyAsync(h_next, m->d_next, M * sizeof(int), cudaMemcpyDeviceToHost, s));
  MS_CUDA(c, cudaMemcpyAsync(h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MS_CUDA(c, cudaStreamSynchronize(s));
  if (*h_err) return check_device_errors(c);
  memcpy(next_ids, h_next, M * sizeof(int));
  return MS_OK;
}

extern "C" ms_status ms_generate(ms_ctx* c, const ms_model* mc, ms_kv* kv, const int* ids,
                                 const int* seq, const int* pos, int M, int steps, int* out_ids,
                                 float* device_ms) {
  if (!c || !mc || !kv || !ids || !out_ids) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  if (steps <= 0) return fail(c, MS_ERR_INVALID_ARG, "steps=%d", steps);
  cudaStream_t s = c->stream;
  if (m->hist_cap < steps * M) {
    cudaStreamSynchronize(s);
    if (m->d_hist) cudaFree(m->d_hist);
    m->d_hist = nullptr;
    m->hist_cap = 0;
    MS_TRY(dev_alloc(c, (void**)&m->d_hist, (size_t)steps * M * sizeof(int)));
    m->hist_cap = steps * M;
  }
  MS_TRY(stage_rows(c, m, kv, ids, seq, pos, M, steps, s));
  MS_TRY(ensure_graph(c, m, kv, M));
  MS_CUDA(c, cudaMemsetAsync(m->d_step, 0, sizeof(int), s));
  MS_CUDA(c, cudaEventRecord(c->ev[0], s));
  for (int i = 0; i < steps; ++i) {
    MS_CUDA(c, cudaGraphLaunch(m->gexec, s));
    MS_CUDA(c, launch_advance_step(m->d_ids, m->d_next, m->d_pos, m->d_hist, m->d_step, M, s, false));
  }
  MS_CUDA(c, cudaEventRecord(c->ev[1], s));
  MS_CUDA(c, cudaMemcpyAsync(out_ids, m->d_hist, (size_t)steps * M * sizeof(int),
                             cudaMemcpyDeviceToHost, s));
  MS_CUDA(c, cudaStreamSynchronize(s));
  if (device_ms) MS_CUDA(c, cudaEventElapsedTime(device_ms, c->ev[0], c->ev[1]));
  return check_device_errors(c);
}

extern "C" void* ms_ctx_stream(ms_ctx* c) { return c ? (void*)c->stream : nullptr; }

// ---------------------------------------------------------------- sampling --

extern "C" ms_status ms_set_sampling(ms_ctx* c, const ms_model* mc, float temperature, float penalty,
                                     uint64_t seed) {
  if (!c || !mc) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  if (m->vocab <= 0) return fail(c, MS_ERR_STATE, "model has no lm_head");
  if (!std::isfinite(temperature) || !std::isfinite(penalty))
    return fail(c, MS_ERR_INVALID_ARG, "temperature %g / penalty %g", temperature, penalty);
  m->samp_t = temperature;
  m->samp_pen = penalty;
  m->samp_seed = seed;
  ++m->samp_ver;  // the captured decode step is rebuilt on its next use
  if (m->sampling()) MS_TRY(ensure_sampler(c, m, 0));
  return MS_OK;
}

extern "C" ms_status ms_sample(ms_ctx* c, const float* logits, int M, int V, const int* hist,
                               const int* hist_off, float temperature, float penalty,
                               const uint64_t* seeds, int* out_ids, void* stream) {
  if (!c || !logits || !out_ids) return MS_ERR_INVALID_ARG;
  if (M <= 0 || M > 65535 || V <= 0) return fail(c, MS_ERR_SHAPE, "sample: M=%d V=%d", M, V);
  const size_t nch = ((size_t)V + kSampChunk - 1) / kSampChunk;
  if (nch > 1024) return fail(c, MS_ERR_SHAPE, "sample: V=%d above %d", V, 1024 * kSampChunk);
  if (!hist != !hist_off) return fail(c, MS_ERR_INVALID_ARG, "sample: hist and hist_off go together");
  if (!std::isfinite(temperature) || !std::isfinite(penalty))
    return fail(c, MS_ERR_INVALID_ARG, "temperature %g / penalty %g", temperature, penalty);
  if (temperature > 0.01f && !seeds) return fail(c, MS_ERR_INVALID_ARG, "sample: seeds needed");
  if (!is_device_ptr(logits) || !is_device_ptr(out_ids) || (hist && !is_device_ptr(hist_off)) ||
      (seeds && temperature > 0.01f && !is_device_ptr(seeds)))
    return fail(c, MS_ERR_INVALID_ARG, "sample: logits, history, seeds and ids must be device memory");
  cudaStream_t s = pick(c, stream);
  if (c->samp_part_n < (size_t)M * nch || c->samp_cnt_n < (size_t)M) {
    MS_CUDA(c, cudaDeviceSynchronize());
    cudaFree(c->samp_part);
    cudaFree(c->samp_cnt);
    c->samp_part = nullptr;
    c->samp_cnt = nullptr;
    c->samp_part_n = c->samp_cnt_n = 0;
    MS_TRY(dev_alloc(c, (void**)&c->samp_part, (size_t)M * nch * sizeof(float2)));
    MS_TRY(dev_alloc(c, (void**)&c->samp_cnt, (size_t)M * sizeof(int)));
    MS_CUDA(c, cudaMemset(c->samp_cnt, 0, (size_t)M * sizeof(int)));
    c->samp_part_n = (size_t)M * nch;
    c->samp_cnt_n = M;
  }
  SampleParams p{};
  p.logits = logits;
  p.ld = V;
  p.M = M;
  p.V = V;
  p.nchunk = (int)nch;
  p.hist = hist;
  p.hist_off = hist_off;
  p.temperature = temperature;
  p.penalty = penalty;
  p.seeds = temperature > 0.01f ? reinterpret_cast<const unsigned long long*>(seeds) : nullptr;
  p.part = c->samp_part;
  p.counter = c->samp_cnt;
  p.tp_world = 1;
  p.out = out_ids;
  MS_CUDA(c, launch_sample(p, s));
  return MS_OK;
}

extern "C" ms_status ms_prefill(ms_ctx* c, const ms_model* mc, ms_kv* kv, const int* ids,
                                const int* seq, const int* pos, int n_tokens, int* first_ids) {
  if (!c || !mc || !kv || !ids || !seq || !pos) return MS_ERR_INVALID_ARG;
  ms_model* m = const_cast<ms_model*>(mc);
  if (m->vocab <= 0) return fail(c, MS_ERR_STATE, "model has no embedding table");
  if (n_tokens <= 0) return fail(c, MS_ERR_INVALID_ARG, "n_tokens=%d", n_tokens);
  cudaStream_t s = c->stream;
  // last row of every sequence (its logits give the first generated token)
  std::vector<int> last_row(kv->n_seq, -1);
  for (int r = 0; r < n_tokens; ++r) {
    if (seq[r] < 0 || seq[r] >= kv->n_seq) return fail(c, MS_ERR_INVALID_ARG, "row %d: sequence %d", r, seq[r]);
    if (last_row[seq[r]] < 0 || pos[r] > pos[last_row[seq[r]]]) last_row[seq[r]] = r;
  }
  std::vector<int> keep_rows;  // rows (global index) whose hidden state feeds the lm_head
  float* keep = nullptr;
  int n_keep = 0;
  for (int s2 = 0; s2 < kv->n_seq; ++s2)
    if (last_row[s2] >= 0) ++n_keep;
  if (n_keep > m->max_rows)
    return fail(c, MS_ERR_CAPACITY, "prefill: %d sequences exceed max_rows %d", n_keep, m->max_rows);
  if (first_ids && n_keep) MS_TRY(dev_alloc(c, (void**)&keep, (size_t)n_keep * m->hidden * sizeof(float)));
  ms_status st = MS_OK;
  int kept = 0;
  std::vector<int> kept_seq;
  for (int r0 = 0; r0 < n_tokens && st == MS_OK; r0 += m->max_rows) {
    const int M = std::min(m->max_rows, n_tokens - r0);
    st = check_rows(c, m, kv, seq + r0, pos + r0, M);
    if (st != MS_OK) break;
    st = kv_prepare(c, kv, seq + r0, pos + r0, M, 0, s);
    if (st != MS_OK) break;
    st = upload_rows(c, m, seq + r0, pos + r0, M, s);
    if (st != MS_OK) break;
    st = embed_ids(c, m, ids + r0, M, m->X[0], s, kv);
    for (int l = 0; l < m->n_layers && st == MS_OK; ++l)
      st = run_layer(c, m, kv, l, M, m->X[0], m->S[0], m->X[1], m->S[1], s, true, true);
    if (st != MS_OK || !first_ids) continue;
    for (int r = r0; r < r0 + M; ++r)
      if (last_row[seq[r]] == r) {
        cudaMemcpyAsync(keep + (size_t)kept * m->hidden, m->X[0] + (size_t)(r - r0) * m->hidden,
                        m->hidden * sizeof(float), cudaMemcpyDeviceToDevice, s);
        kept_seq.push_back(seq[r]);
        ++kept;
      }
  }
  if (st == MS_OK && first_ids && n_keep) {
    // (errors go through st from here on, so `keep` is always freed below)
    const cudaError_t e = launch_rowstats(m->S[1], keep, m->hidden, n_keep, m->hidden, s, false);
    if (e != cudaSuccess) st = fail(c, MS_ERR_CUDA, "prefill row statistics: %s", cudaGetErrorString(e));
    if (st == MS_OK && m->sampling()) {  // each sequence's last row: its sequence and position
      std::vector<int> ks(kept_seq), kp(n_keep);
      for (int i = 0; i < n_keep; ++i) kp[i] = pos[last_row[kept_seq[i]]];
      st = ensure_sampler(c, m, n_keep);
      if (st == MS_OK) {
        cudaMemcpyAsync(m->d_seq, ks.data(), n_keep * sizeof(int), cudaMemcpyHostToDevice, s);
        cudaMemcpyAsync(m->d_pos, kp.data(), n_keep * sizeof(int), cudaMemcpyHostToDevice, s);
        st = lm_head_launch(c, m, keep, m->S[1], n_keep, m->d_logits, nullptr, s, true);
      }
      if (st == MS_OK) st = sample_rows(c, m, kv, n_keep, m->d_seq, m->d_pos, m->d_next, s);
    } else if (st == MS_OK) {
      st = lm_head_launch(c, m, keep, m->S[1], n_keep, nullptr, m->d_next, s, true);
    }
    std::vector<int> nxt(n_keep);
    if (st == MS_OK) {
      cudaMemcpyAsync(nxt.data(), m->d_next, n_keep * sizeof(int), cudaMemcpyDeviceToHost, s);
      if (cudaStreamSynchronize(s) != cudaSuccess) st = fail(c, MS_ERR_CUDA, "prefill sync");
    }
    if (st == MS_OK)
      for (int i = 0; i < n_keep; ++i) first_ids[kept_seq[i]] = nxt[i];
  }
  if (keep) {
    cudaStreamSynchronize(s);
    cudaFree(keep);
  }
  if (st == MS_OK) MS_CUDA(c, cudaStreamSynchronize(s));
  if (st == MS_OK) st = check_device_errors(c);
  return st;
}
