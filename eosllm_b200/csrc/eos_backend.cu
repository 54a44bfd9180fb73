// eos_backend.cu -- the C ABI of libeosllm_cuda.so (include/eosllm_cuda.h).
//
// Host-pointer layer: the semantics of the reference backend slot
// eos_backend_ops_t.matmul_q (include/eosllm/backend.h:43-46) -- synchronous,
// caller-owned host buffers, status codes instead of aborts, outputs written
// only on success.  Weights are uploaded on first use into a per-device cache
// keyed by (host pointer, dtype, n, k) plus a 128-byte fingerprint, and the
// n output rows are split across the selected GPUs (rows are independent,
// src/kernels/avx2/matmul_q4_k_int8.c:215-265): every GPU gets the whole A,
// computes its row range into its own buffer, and the slices land in
// disjoint columns of the pinned host output -- no collective is needed.
//
// Device-pointer layer: enqueue-only wrappers around the same launchers.
#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "eosllm_cuda.h"
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace {

thread_local char g_err[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear the sticky-free error state
  return fail(e == cudaErrorMemoryAllocation ? EOS_E_OUT_OF_MEMORY : EOS_E_INTERNAL, "%s: %s (%s)", what,
              cudaGetErrorString(e), cudaGetErrorName(e));
}

#define EOS_CK(call, what)                           \
  do {                                               \
    cudaError_t e_ = (call);                         \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// ---- per-device facts and error words (both layers) ----------------------
struct DevInfo {
  bool ready = false;
  int num_sms = 0;
  int max_smem = 0;
  uint32_t* err_d = nullptr;  // device word the kernels OR error bits into
};

std::mutex g_info_mu;
// One entry per device ordinal, never moved: shards and callers keep
// pointers to their device's entry.
DevInfo g_info[eos::kMaxDevices];

int device_info(int dev, DevInfo** out) {
  std::lock_guard<std::mutex> lk(g_info_mu);
  if (dev < 0 || dev >= eos::kMaxDevices) return fail(EOS_E_INVALID_ARG, "bad device %d", dev);
  DevInfo& d = g_info[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    EOS_CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "cudaDeviceGetAttribute");
    EOS_CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev), "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
      return fail(EOS_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                  minor);
    EOS_CK(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
    EOS_CK(cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
           "cudaDeviceGetAttribute");
    int cur = 0;
    EOS_CK(cudaGetDevice(&cur), "cudaGetDevice");
    EOS_CK(cudaSetDevice(dev), "cudaSetDevice");
    cudaError_t e = cudaMalloc(&d.err_d, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(d.err_d, 0, sizeof(uint32_t));
    cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "error word");
    d.ready = true;
  }
  *out = &d;
  return EOS_OK;
}


// ---- host-pointer layer state ---------------------------------------------
struct WeightEntry {
  uint8_t* dev = nullptr;  // this device's row shard
  size_t bytes = 0;
  uint8_t fp[128];
};

struct Key {
  const void* host;
  int dtype;
  uint32_t n, k;
  bool operator==(const Key& o) const { return host == o.host && dtype == o.dtype && n == o.n && k == o.k; }
};
struct KeyHash {
  size_t operator()(const Key& x) const {
    return std::hash<const void*>()(x.host) ^ ((size_t)x.n * 1000003u) ^ ((size_t)x.k << 20) ^ (size_t)x.dtype;
  }
};

// The launches of one host-pointer Q4_K call (packing, GEMVs, copy-out,
// done flag), recorded once as a CUDA graph per weight slice, shape and
// buffer set: every later call with the same key is one cudaGraphLaunch.
struct GKey {
  const void* w;
  const void* a;
  const void* act;
  const void* c;
  const void* blk;
  uint32_t m, rows, k;
  bool operator==(const GKey& o) const {
    return w == o.w && a == o.a && act == o.act && c == o.c && blk == o.blk && m == o.m && rows == o.rows && k == o.k;
  }
};
struct GKeyHash {
  size_t operator()(const GKey& x) const {
    return std::hash<const void*>()(x.w) ^ (std::hash<const void*>()(x.a) << 1) ^ ((size_t)x.m * 131u) ^
           ((size_t)x.rows * 1000003u) ^ ((size_t)x.k << 24);
  }
};
constexpr size_t kMaxCallGraphs = 1024;

struct Shard {
  int dev = -1;
  DevInfo* info = nullptr;
  cudaStream_t stream = nullptr;
  float* d_a = nullptr;
  size_t cap_a = 0;
  float* d_c = nullptr;
  size_t cap_c = 0;
  uint8_t* d_act = nullptr;
  size_t cap_act = 0;
  uint32_t* h_err = nullptr;  // pinned copy of the error word
  uint8_t* h_blk = nullptr;      // mapped pinned: Q4_K path's status header + outputs
  uint8_t* h_blk_dev = nullptr;  // its device alias, written by copy_out_kernel
  size_t cap_blk = 0;
  std::unordered_map<Key, WeightEntry, KeyHash> cache;
  std::unordered_map<GKey, cudaGraphExec_t, GKeyHash> graphs;
};

void drop_graphs(Shard& s) {
  for (auto& kv : s.graphs) cudaGraphExecDestroy(kv.second);
  s.graphs.clear();
}

std::recursive_mutex g_mu;
std::vector<Shard> g_shards;
bool g_host_ready = false;
std::vector<int> g_requested;  // from eosi_cuda_set_devices
float* g_h_a = nullptr;
size_t g_cap_h_a = 0;
float* g_h_c = nullptr;
size_t g_cap_h_c = 0;

int g_probe = -1;
int g_ndev = 0;
uint64_t g_host_calls = 0;  // host-pointer matmuls completed on the GPU

size_t row_bytes_of(int dtype, uint32_t k) {
  return dtype == EOS_DT_Q4_K ? (size_t)(k / Q4K_ELEMS) * Q4K_BYTES : (size_t)(k / Q80_ELEMS) * Q80_BYTES;
}

void fingerprint(const void* host, size_t bytes, uint8_t out[128]) {
  memset(out, 0, 128);
  const size_t h = bytes < 64 ? bytes : 64;
  memcpy(out, host, h);
  memcpy(out + 64, (const uint8_t*)host + (bytes - h), h);
}

void release_shard(Shard& s) {
  if (s.dev < 0) return;
  cudaSetDevice(s.dev);
  drop_graphs(s);
  for (auto& kv : s.cache) cudaFree(kv.second.dev);
  s.cache.clear();
  cudaFree(s.d_a);
  cudaFree(s.d_c);
  cudaFree(s.d_act);
  if (s.h_err) cudaFreeHost(s.h_err);
  if (s.h_blk) cudaFreeHost(s.h_blk);
  if (s.stream) cudaStreamDestroy(s.stream);
  s = Shard();
}

void release_all() {
  int prev = 0;
  const bool had = cudaGetDevice(&prev) == cudaSuccess;
  for (auto& s : g_shards) release_shard(s);
  if (had) cudaSetDevice(prev);  // the caller's current device, as found
  g_shards.clear();
  if (g_h_a) cudaFreeHost(g_h_a);
  if (g_h_c) cudaFreeHost(g_h_c);
  g_h_a = g_h_c = nullptr;
  g_cap_h_a = g_cap_h_c = 0;
  g_host_ready = false;
}

std::vector<int> default_devices() {
  std::vector<int> ids;
  if (const char* env = getenv("EOSLLM_CUDA_DEVICES")) {
    const char* p = env;
    while (*p) {
      char* endp = nullptr;
      long v = strtol(p, &endp, 10);
      if (endp == p) break;
      ids.push_back((int)v);
      p = endp;
      while (*p == ',' || *p == ' ') ++p;
    }
  }
  if (ids.empty()) ids.push_back(0);
  return ids;
}

int host_init() {
  if (g_host_ready) return EOS_OK;
  if (eosi_cuda_probe() != EOS_OK) return fail(EOS_E_UNSUPPORTED, "no usable sm_100 GPU: %s", g_err);
  std::vector<int> ids = g_requested.empty() ? default_devices() : g_requested;
  int prev = 0;
  cudaGetDevice(&prev);
  for (int id : ids) {
    if (id < 0 || id >= g_ndev) {
      release_all();
      return fail(EOS_E_INVALID_ARG, "device %d out of range (0..%d)", id, g_ndev - 1);
    }
    Shard s;
    s.dev = id;
    int rc = device_info(id, &s.info);
    if (rc != EOS_OK) {
      release_all();
      return rc;
    }
    cudaSetDevice(id);
    cudaError_t e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc(&s.h_err, sizeof(uint32_t), cudaHostAllocDefault);
    if (e != cudaSuccess) {
      g_shards.push_back(s);
      release_all();
      cudaSetDevice(prev);
      return cuda_fail(e, "backend init");
    }
    *s.h_err = 0;
    g_shards.push_back(s);
  }
  cudaSetDevice(prev);
  g_host_ready = true;
  return EOS_OK;
}

template <typename T>
int ensure_dev(T** p, size_t* cap, size_t bytes, const char* what) {
  if (*cap >= bytes) return EOS_OK;
  cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t want = std::max(bytes, (size_t)4096);
  EOS_CK(cudaMalloc(p, want), what);
  *cap = want;
  return EOS_OK;
}

int ensure_pinned(float** p, size_t* cap, size_t bytes) {
  if (*cap >= bytes) return EOS_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  size_t want = std::max(bytes, (size_t)65536);
  // portable (every device's context treats it as pinned) and mapped (a
  // kernel may read it directly: the Q4_K path's activations)
  EOS_CK(cudaHostAlloc((void**)p, want, cudaHostAllocPortable | cudaHostAllocMapped), "pinned staging");
  *cap = want;
  return EOS_OK;
}

// Device copy of rows [row0, row0 + rows) of one host weight buffer.
int cached_weight(Shard& s, const void* host, int dtype, uint32_t n, uint32_t k, uint32_t row0, uint32_t rows,
                  uint8_t** out) {
  const size_t rb = row_bytes_of(dtype, k);
  const size_t total = rb * n;
  Key key{host, dtype, n, k};
  uint8_t fp[128];
  fingerprint(host, total, fp);
  auto it = s.cache.find(key);
  if (it != s.cache.end()) {
    if (memcmp(it->second.fp, fp, 128) == 0) {
      *out = it->second.dev;
      return EOS_OK;
    }
    cudaFree(it->second.dev);
    s.cache.erase(it);
  }
  WeightEntry e;
  e.bytes = rb * rows;
  memcpy(e.fp, fp, 128);
  EOS_CK(cudaMalloc(&e.dev, std::max(e.bytes, (size_t)16)), "weight upload (cudaMalloc)");
  cudaError_t ce = cudaMemcpy(e.dev, (const uint8_t*)host + rb * row0, e.bytes, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) {
    cudaFree(e.dev);
    return cuda_fail(ce, "weight upload (cudaMemcpy)");
  }
  s.cache.emplace(key, e);
  *out = e.dev;
  return EOS_OK;
}

// Enqueue C[m, rows] = A . deq(W_shard)^T on one device.  `n_total` decides
// the Q4_K small-n path exactly as the reference does (on the full n).
int enqueue_matmul(DevInfo* info, int dtype, const float* d_a, const uint8_t* d_w, float* d_c, uint32_t m,
                   uint32_t rows, uint32_t n_total, uint32_t k, uint8_t* d_act, cudaStream_t st) {
  if (rows == 0 || m == 0) return EOS_OK;
  if (dtype == EOS_DT_Q4_K) {
    if (n_total < 4) {
      EOS_CK(eos::launch_q4k_f32_small_n(d_a, d_w, d_c, m, rows, k, st), "q4_k small-n kernel");
      return EOS_OK;
    }
    if (m == 1 && d_act == nullptr) {  // no scratch: activation packing fused into the GEMV
      int status = EOS_OK;
      EOS_CK(eos::launch_q4k_gemv(d_w, nullptr, d_a, d_c, rows, k, info->err_d, info->num_sms, info->max_smem, true,
                                  st, &status),
             "q4_k gemv kernel");
      if (status == EOS_OK) return EOS_OK;
      if (d_act == nullptr) return fail(EOS_E_INVALID_ARG, "q4_k: k=%u needs the scratch buffer", k);
    }
    if (d_act == nullptr) return fail(EOS_E_INVALID_ARG, "NULL scratch");
    EOS_CK(eos::launch_act_pack(d_a, m, k, d_act, EOS_ACT_LAYOUT_GEMV, st), "activation pack kernel");
    const size_t act_stride = eos::act_layout_bytes(1, k, EOS_ACT_LAYOUT_GEMV);
    for (uint32_t i = 0; i < m; ++i) {
      int status = EOS_OK;
      EOS_CK(eos::launch_q4k_gemv(d_w, d_act + i * act_stride, nullptr, d_c + (size_t)i * rows, rows, k,
                                  info->err_d, info->num_sms, info->max_smem, true, st, &status),
             "q4_k gemv kernel");
      if (status != EOS_OK) return fail(status, "q4_k gemv: shape %u x %u not supported", rows, k);
    }
    return EOS_OK;
  }
  // Q8_0
  for (uint32_t i = 0; i < m; ++i) {
    int status = EOS_OK;
    EOS_CK(eos::launch_q80_gemv(d_w, d_a + (size_t)i * k, d_c + (size_t)i * rows, rows, k, info->err_d,
                                info->num_sms, info->max_smem, st, &status),
           "q8_0 gemv kernel");
    if (status != EOS_OK) return fail(status, "q8_0 gemv: shape %u x %u not supported", rows, k);
  }
  return EOS_OK;
}

int check_args(const void* a, const void* b, const void* c, int dtype, uint32_t k) {
  if (a == nullptr || b == nullptr || c == nullptr) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (dtype == EOS_DT_Q4_K) {
    if (k % Q4K_ELEMS) return fail(EOS_E_INVALID_ARG, "q4_k: k=%u is not a multiple of 256", k);
  } else if (dtype == EOS_DT_Q8_0) {
    if (k % Q80_ELEMS) return fail(EOS_E_INVALID_ARG, "q8_0: k=%u is not a multiple of 32", k);
  } else {
    return fail(EOS_E_UNSUPPORTED, "dtype %d not supported by the cuda backend", dtype);
  }
  return EOS_OK;
}

int host_matmul(const float* a, const void* b, int dtype, float* c, uint32_t m, uint32_t n, uint32_t k) {
  int rc = check_args(a, b, c, dtype, k);
  if (rc != EOS_OK) return rc;
  if (m == 0 || n == 0) return EOS_OK;
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  rc = host_init();
  if (rc != EOS_OK) return rc;
  const uint32_t G = (uint32_t)g_shards.size();
  rc = ensure_pinned(&g_h_a, &g_cap_h_a, (size_t)m * k * 4u);
  if (rc == EOS_OK) rc = ensure_pinned(&g_h_c, &g_cap_h_c, (size_t)m * n * 4u);
  if (rc != EOS_OK) return rc;
  int prev = 0;
  cudaGetDevice(&prev);
  memcpy(g_h_a, a, (size_t)m * k * 4u);
  std::vector<char> used(G, 0);
  std::vector<volatile uint32_t*> flags(G, nullptr);  // Q4_K path: each shard's done flag
  // Q4_K with n >= 4 (the int8 path): zero-copy activations and outputs
  const bool q4k_fast = dtype == EOS_DT_Q4_K && n >= 4;
  const float* d_a_mapped = nullptr;
  if (q4k_fast) {
    void* dp = nullptr;
    EOS_CK(cudaHostGetDevicePointer(&dp, g_h_a, 0), "mapped activations");
    d_a_mapped = static_cast<const float*>(dp);
  }
  for (uint32_t gi = 0; gi < G && rc == EOS_OK; ++gi) {
    Shard& s = g_shards[gi];
    const uint32_t row0 = (uint32_t)(((uint64_t)n * gi) / G), row1 = (uint32_t)(((uint64_t)n * (gi + 1)) / G);
    const uint32_t rows = row1 - row0;
    if (rows == 0) continue;
    if (cudaSetDevice(s.dev) != cudaSuccess) {
      rc = cuda_fail(cudaGetLastError(), "cudaSetDevice");
      break;
    }
    uint8_t* d_w = nullptr;
    rc = cached_weight(s, b, dtype, n, k, row0, rows, &d_w);
    if (rc == EOS_OK) rc = ensure_dev(&s.d_a, &s.cap_a, (size_t)m * k * 4u, "activation buffer");
    if (rc == EOS_OK) rc = ensure_dev(&s.d_c, &s.cap_c, (size_t)m * rows * 4u, "output buffer");
    if (rc == EOS_OK && dtype == EOS_DT_Q4_K)
      rc = ensure_dev(&s.d_act, &s.cap_act, eos::act_layout_bytes(m, k, EOS_ACT_LAYOUT_GEMV), "act scratch");
    if (rc != EOS_OK) break;
    if (q4k_fast) {
      // Q4_K: the packing kernel reads the activations straight from the
      // mapped pinned staging buffer (no H2D copy) and zeroes a status word
      // the GEMVs report into; a copy kernel chained behind the GEMVs writes
      // status word + outputs into mapped pinned memory (no copy engine)
      const size_t blk = 16u + (((size_t)m * rows * 4u + 15u) & ~(size_t)15u);
      rc = ensure_dev(&s.d_c, &s.cap_c, blk, "output buffer");
      // the done flag sits just past the copied block (its own 16 bytes)
      if (rc == EOS_OK && s.cap_blk < blk + 16u) {
        if (s.h_blk) cudaFreeHost(s.h_blk);
        s.h_blk = nullptr;
        s.h_blk_dev = nullptr;
        s.cap_blk = 0;
        const size_t want = std::max(blk + 16u, (size_t)65536);
        cudaError_t ae = cudaHostAlloc((void**)&s.h_blk, want, cudaHostAllocPortable | cudaHostAllocMapped);
        void* dp = nullptr;
        if (ae == cudaSuccess) ae = cudaHostGetDevicePointer(&dp, s.h_blk, 0);
        if (ae != cudaSuccess) {
          if (s.h_blk) cudaFreeHost(s.h_blk);
          s.h_blk = nullptr;
          rc = cuda_fail(ae, "pinned output staging");
        } else {
          s.h_blk_dev = static_cast<uint8_t*>(dp);
          s.cap_blk = want;
        }
      }
      if (rc != EOS_OK) break;
      used[gi] = 1;
      uint32_t* status = reinterpret_cast<uint32_t*>(s.d_c);
      float* d_out = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d_c) + 16);
      const GKey gk{d_w, d_a_mapped, s.d_act, s.d_c, s.h_blk_dev, m, rows, k};
      auto git = s.graphs.find(gk);
      if (git == s.graphs.end()) {
        // record the call's launches once: packing (zeroes the status word),
        // the GEMVs, the copy of status word + outputs into mapped memory,
        // then the done flag (word 1 of the block)
        if (s.graphs.size() >= kMaxCallGraphs) drop_graphs(s);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeRelaxed);
        cudaError_t le = cudaSuccess;
        int st2 = EOS_OK;
        if (e == cudaSuccess) {
          le = eos::launch_act_pack(d_a_mapped, m, k, s.d_act, EOS_ACT_LAYOUT_GEMV, s.stream, status);
          const size_t act_stride = eos::act_layout_bytes(1, k, EOS_ACT_LAYOUT_GEMV);
          for (uint32_t i = 0; i < m && le == cudaSuccess && st2 == EOS_OK; ++i)
            le = eos::launch_q4k_gemv(d_w, s.d_act + i * act_stride, nullptr, d_out + (size_t)i * rows, rows, k,
                                      status, s.info->num_sms, s.info->max_smem, true, s.stream, &st2);
          if (le == cudaSuccess) le = eos::launch_copy_out(s.d_c, s.h_blk_dev, blk, s.stream);
          if (le == cudaSuccess) le = eos::launch_done_flag(reinterpret_cast<uint32_t*>(s.h_blk_dev + blk), s.stream);
          e = cudaStreamEndCapture(s.stream, &g);
          if (le != cudaSuccess) e = le;
        }
        cudaGraphExec_t ge = nullptr;
        if (e == cudaSuccess && st2 == EOS_OK) e = cudaGraphInstantiate(&ge, g, 0);
        if (g) cudaGraphDestroy(g);
        if (e != cudaSuccess) {
          rc = cuda_fail(e, "q4_k call graph");
          break;
        }
        if (st2 != EOS_OK) {
          rc = fail(st2, "q4_k gemv: shape %u x %u not supported", rows, k);
          break;
        }
        git = s.graphs.emplace(gk, ge).first;
      }
      flags[gi] = reinterpret_cast<volatile uint32_t*>(s.h_blk + blk);
      *flags[gi] = 0u;  // the done flag, raised by the graph's last node
      const cudaError_t e = cudaGraphLaunch(git->second, s.stream);
      if (e != cudaSuccess) rc = cuda_fail(e, "q4_k call graph launch");
      continue;
    }
    cudaError_t e = cudaMemcpyAsync(s.d_a, g_h_a, (size_t)m * k * 4u, cudaMemcpyHostToDevice, s.stream);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "H2D activations");
      break;
    }
    used[gi] = 1;
    rc = enqueue_matmul(s.info, dtype, s.d_a, d_w, s.d_c, m, rows, n, k, s.d_act, s.stream);
    if (rc != EOS_OK) break;
    e = cudaMemcpy2DAsync(g_h_c + row0, (size_t)n * 4u, s.d_c, (size_t)rows * 4u, (size_t)rows * 4u, m,
                          cudaMemcpyDeviceToHost, s.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s.h_err, s.info->err_d, 4, cudaMemcpyDeviceToHost, s.stream);
    if (e != cudaSuccess) rc = cuda_fail(e, "D2H outputs");
  }
  // Always drain every stream we used, even after a failure.  The Q4_K path
  // waits for its done flag in mapped memory (bounded), and synchronises the
  // stream only when it does not come (an error then surfaces there).
  for (uint32_t gi = 0; gi < G; ++gi) {
    if (!used[gi]) continue;
    Shard& s = g_shards[gi];
    cudaSetDevice(s.dev);
    bool flagged = false;
    if (q4k_fast && rc == EOS_OK && flags[gi] != nullptr) {
      const volatile uint32_t* flag = flags[gi];
      const auto t0 = std::chrono::steady_clock::now();
      for (uint32_t spin = 0;; ++spin) {
        if (*flag != 0u) {
          flagged = true;
          break;
        }
        if ((spin & 1023u) == 1023u && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2)) break;
      }
    }
    cudaError_t e = flagged ? cudaSuccess : cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess && rc == EOS_OK) rc = cuda_fail(e, "kernel execution");
    const uint32_t bits = q4k_fast ? *reinterpret_cast<const uint32_t*>(s.h_blk) : *s.h_err;
    if (rc == EOS_OK && bits != 0) {
      if (!q4k_fast) {
        *s.h_err = 0;
        cudaMemset(s.info->err_d, 0, 4);
      }
      rc = fail(EOS_E_INTERNAL, "device %d: bounded wait gave up (error bits 0x%x)", s.dev, bits);
    }
  }
  cudaSetDevice(prev);
  if (rc != EOS_OK) return rc;
  if (q4k_fast) {  // each shard's rows into c (written only on success)
    for (uint32_t gi = 0; gi < G; ++gi) {
      if (!used[gi]) continue;
      const uint32_t row0 = (uint32_t)(((uint64_t)n * gi) / G), row1 = (uint32_t)(((uint64_t)n * (gi + 1)) / G);
      const uint32_t rows = row1 - row0;
      const float* src = reinterpret_cast<const float*>(g_shards[gi].h_blk + 16);
      for (uint32_t i = 0; i < m; ++i) memcpy(c + (size_t)i * n + row0, src + (size_t)i * rows, (size_t)rows * 4u);
    }
    ++g_host_calls;
    return EOS_OK;
  }
  memcpy(c, g_h_c, (size_t)m * n * 4u);
  ++g_host_calls;
  return EOS_OK;
}

// A *_dev entry point runs on the caller's current device, so every pointer
// it is given must be device (or managed) memory of that device: a host
// pointer or another GPU's memory is rejected here instead of being handed
// to a kernel.
int check_on_device(const void* p, int dev) {
  if (p == nullptr) return EOS_OK;
  cudaPointerAttributes at;
  const cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(EOS_E_INVALID_ARG, "pointer %p is not CUDA memory", p);
  }
  if (at.type == cudaMemoryTypeManaged) return EOS_OK;
  if (at.type != cudaMemoryTypeDevice)
    return fail(EOS_E_INVALID_ARG, "pointer %p is host memory; the *_dev entry points take device pointers", p);
  if (at.device != dev)
    return fail(EOS_E_INVALID_ARG, "pointer %p is on device %d, the current device is %d", p, at.device, dev);
  return EOS_OK;
}

int dev_prologue(DevInfo** info, std::initializer_list<const void*> ptrs = {}) {
  if (eosi_cuda_probe() != EOS_OK) return fail(EOS_E_UNSUPPORTED, "no usable sm_100 GPU");
  int dev = 0;
  EOS_CK(cudaGetDevice(&dev), "cudaGetDevice");
  int rc = device_info(dev, info);
  for (const void* p : ptrs)
    if (rc == EOS_OK) rc = check_on_device(p, dev);
  return rc;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace eos {
void set_error_message(const char* msg) { fail(EOS_OK, "%s", msg); }
int pointers_on_device(std::initializer_list<const void*> ptrs, int dev) {
  for (const void* p : ptrs) {
    const int rc = check_on_device(p, dev);
    if (rc != EOS_OK) return rc;
  }
  return EOS_OK;
}
}  // namespace eos

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int eosi_cuda_probe(void) {
  if (g_probe >= 0) return g_probe;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n <= 0) {
    cudaGetLastError();
    g_ndev = 0;
    g_probe = EOS_E_UNSUPPORTED;
    fail(EOS_E_UNSUPPORTED, "no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
    return g_probe;
  }
  int ok = 0;
  for (int d = 0; d < n; ++d) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d);
    if (major == 10 && minor == 0) ++ok;
  }
  g_ndev = n;
  g_probe = ok > 0 ? EOS_OK : EOS_E_UNSUPPORTED;
  if (!ok) fail(EOS_E_UNSUPPORTED, "no sm_100 device among %d", n);
  return g_probe;
}

int eosi_cuda_device_count(void) {
  if (eosi_cuda_probe() != EOS_OK) return 0;
  int ok = 0;
  for (int d = 0; d < g_ndev; ++d) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d);
    if (major == 10 && minor == 0) ++ok;
  }
  return ok;
}

int eosi_cuda_set_devices(const int* ids, int count) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  release_all();
  g_requested.clear();
  if (ids != nullptr && count > 0) g_requested.assign(ids, ids + count);
  return EOS_OK;
}

void eosi_cuda_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  release_all();
  std::lock_guard<std::mutex> lk2(g_info_mu);
  int prev = 0;
  const bool had = cudaGetDevice(&prev) == cudaSuccess;
  for (int d = 0; d < eos::kMaxDevices; ++d)
    if (g_info[d].err_d) {
      cudaSetDevice(d);
      cudaFree(g_info[d].err_d);
      g_info[d] = DevInfo();
    }
  if (had) cudaSetDevice(prev);
}

const char* eosi_cuda_last_error(void) { return g_err; }

int eosi_cuda_matmul_q(const float* a, const void* b_quant, int b_dtype, float* c, uint32_t m, uint32_t n,
                       uint32_t k) {
  return host_matmul(a, b_quant, b_dtype, c, m, n, k);
}

int eosi_cuda_matmul_q4_k(const float* a, const void* b_q4, float* c, uint32_t m, uint32_t n, uint32_t k) {
  return host_matmul(a, b_q4, EOS_DT_Q4_K, c, m, n, k);
}

int eosi_cuda_matmul_q8_0(const float* a, const void* b_q8, float* c, uint32_t m, uint32_t n, uint32_t k) {
  return host_matmul(a, b_q8, EOS_DT_Q8_0, c, m, n, k);
}

int eosi_cuda_cache_evict(const void* b_quant) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int prev = 0;  // the caller's device is current again on return
  const bool had = cudaGetDevice(&prev) == cudaSuccess;
  for (auto& s : g_shards) {
    cudaSetDevice(s.dev);
    drop_graphs(s);  // they may reference the evicted weights
    for (auto it = s.cache.begin(); it != s.cache.end();) {
      if (it->first.host == b_quant) {
        cudaFree(it->second.dev);
        it = s.cache.erase(it);
      } else {
        ++it;
      }
    }
  }
  if (had) cudaSetDevice(prev);
  return EOS_OK;
}

int eosi_cuda_cache_clear(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int prev = 0;  // the caller's device is current again on return
  const bool had = cudaGetDevice(&prev) == cudaSuccess;
  for (auto& s : g_shards) {
    cudaSetDevice(s.dev);
    drop_graphs(s);
    for (auto& kv : s.cache) cudaFree(kv.second.dev);
    s.cache.clear();
  }
  if (had) cudaSetDevice(prev);
  return EOS_OK;
}

int eosi_cuda_host_stats(uint64_t* calls, uint64_t* cached_weights, uint64_t* cached_bytes) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  uint64_t entries = 0, bytes = 0;
  for (const auto& s : g_shards)
    for (const auto& kv : s.cache) {
      ++entries;
      bytes += kv.second.bytes;
    }
  if (calls) *calls = g_host_calls;
  if (cached_weights) *cached_weights = entries;
  if (cached_bytes) *cached_bytes = bytes;
  return EOS_OK;
}

int eosi_cuda_cache_preload(const void* b_quant, int b_dtype, uint32_t n, uint32_t k) {
  float dummy = 0.0f;
  int rc = check_args(&dummy, b_quant, &dummy, b_dtype, k);
  if (rc != EOS_OK) return rc;
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  rc = host_init();
  if (rc != EOS_OK) return rc;
  const uint32_t G = (uint32_t)g_shards.size();
  int prev = 0;
  cudaGetDevice(&prev);
  for (uint32_t gi = 0; gi < G && rc == EOS_OK; ++gi) {
    const uint32_t row0 = (uint32_t)(((uint64_t)n * gi) / G), row1 = (uint32_t)(((uint64_t)n * (gi + 1)) / G);
    if (row1 == row0) continue;
    cudaSetDevice(g_shards[gi].dev);
    uint8_t* d = nullptr;
    rc = cached_weight(g_shards[gi], b_quant, b_dtype, n, k, row0, row1 - row0, &d);
  }
  cudaSetDevice(prev);
  return rc;
}

size_t eosi_cuda_q4_k_scratch_bytes(uint32_t m, uint32_t k) {
  return eos::act_layout_bytes(m, k, EOS_ACT_LAYOUT_GEMV);
}

int eosi_cuda_matmul_q4_k_dev(const float* a, const void* w, float* c, uint32_t m, uint32_t n, uint32_t k,
                              void* scratch, void* stream) {
  int rc = check_args(a, w, c, EOS_DT_Q4_K, k);
  if (rc != EOS_OK) return rc;
  if (!al16(a) || !al16(w) || (scratch && !al16(scratch)))
    return fail(EOS_E_INVALID_ARG, "device pointers must be 16-byte aligned");
  if (m == 0 || n == 0) return EOS_OK;
  DevInfo* info = nullptr;
  rc = dev_prologue(&info, {a, w, c, scratch});
  if (rc != EOS_OK) return rc;
  return enqueue_matmul(info, EOS_DT_Q4_K, a, (const uint8_t*)w, c, m, n, n, k, (uint8_t*)scratch,
                        (cudaStream_t)stream);
}

int eosi_cuda_q4_k_pack_act_dev(const float* a, uint32_t m, uint32_t k, void* act, void* stream) {
  if (a == nullptr || act == nullptr) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (k % Q4K_ELEMS) return fail(EOS_E_INVALID_ARG, "q4_k: k=%u is not a multiple of 256", k);
  if (!al16(act)) return fail(EOS_E_INVALID_ARG, "act must be 16-byte aligned");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {a, act});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_act_pack(a, m, k, (uint8_t*)act, EOS_ACT_LAYOUT_GEMV, (cudaStream_t)stream),
         "activation pack kernel");
  return EOS_OK;
}

int eosi_cuda_q4_k_gemv_dev(const void* act, const void* w, float* c, uint32_t n, uint32_t k, void* stream) {
  int rc = check_args(act, w, c, EOS_DT_Q4_K, k);
  if (rc != EOS_OK) return rc;
  if (!al16(act) || !al16(w)) return fail(EOS_E_INVALID_ARG, "device pointers must be 16-byte aligned");
  DevInfo* info = nullptr;
  rc = dev_prologue(&info, {act, w, c});
  if (rc != EOS_OK) return rc;
  int status = EOS_OK;
  EOS_CK(eos::launch_q4k_gemv((const uint8_t*)w, (const uint8_t*)act, nullptr, c, n, k, info->err_d, info->num_sms,
                              info->max_smem, true, (cudaStream_t)stream, &status),
         "q4_k gemv kernel");
  if (status != EOS_OK) return fail(status, "q4_k gemv: shape %u x %u not supported", n, k);
  return EOS_OK;
}

size_t eosi_cuda_q4_k_prefill_weight_bytes(uint32_t n, uint32_t k) { return eos::prefill_operand_bytes(n, k); }

size_t eosi_cuda_q4_k_prefill_scratch_bytes(uint32_t m, uint32_t k) { return eos::prefill_operand_bytes(m, k); }

int eosi_cuda_q4_k_prefill_prepare_weights_dev(const void* w, uint32_t n, uint32_t k, void* w_prep, void* stream) {
  int rc = check_args(w, w_prep, w_prep, EOS_DT_Q4_K, k);
  if (rc != EOS_OK) return rc;
  if (!al16(w) || !al16(w_prep)) return fail(EOS_E_INVALID_ARG, "prefill weights must be 16-byte aligned");
  DevInfo* info = nullptr;
  rc = dev_prologue(&info, {w, w_prep});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_prefill_w_prep((const uint8_t*)w, n, k, w_prep, (cudaStream_t)stream), "prefill weight prep");
  return EOS_OK;
}

int eosi_cuda_q4_k_prefill_dev(const float* a, const void* w_prep, float* c, uint32_t m, uint32_t n, uint32_t k,
                               void* scratch, void* stream) {
  int rc = check_args(a, w_prep, c, EOS_DT_Q4_K, k);
  if (rc != EOS_OK) return rc;
  if (scratch == nullptr) return fail(EOS_E_INVALID_ARG, "NULL scratch pointer");
  if (!al16(a) || !al16(w_prep) || !al16(scratch) || !al16(c))
    return fail(EOS_E_INVALID_ARG, "prefill pointers must be 16-byte aligned");
  if (m == 0 || n == 0) return EOS_OK;
  DevInfo* info = nullptr;
  rc = dev_prologue(&info, {a, w_prep, c, scratch});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_prefill_act_pack(a, m, k, scratch, (cudaStream_t)stream), "prefill activation packing");
  int status = EOS_OK;
  EOS_CK(eos::launch_prefill_gemm(scratch, w_prep, c, m, n, k, info->err_d, (cudaStream_t)stream, &status),
         "prefill gemm");
  if (status != EOS_OK) return fail(status, "prefill gemm: tensor maps unavailable for %u x %u x %u", m, n, k);
  return EOS_OK;
}

int eosi_cuda_matmul_q8_0_dev(const float* a, const void* w, float* c, uint32_t m, uint32_t n, uint32_t k,
                              void* stream) {
  int rc = check_args(a, w, c, EOS_DT_Q8_0, k);
  if (rc != EOS_OK) return rc;
  if (!al16(a)) return fail(EOS_E_INVALID_ARG, "activations must be 16-byte aligned");
  if (m == 0 || n == 0) return EOS_OK;
  DevInfo* info = nullptr;
  rc = dev_prologue(&info, {a, w, c});
  if (rc != EOS_OK) return rc;
  return enqueue_matmul(info, EOS_DT_Q8_0, a, (const uint8_t*)w, c, m, n, n, k, nullptr, (cudaStream_t)stream);
}

int eosi_cuda_quantize_act_dev(const float* a, uint32_t m, uint32_t k, int8_t* aq, float* scales, int32_t* sums,
                               void* stream) {
  if (!a || !aq || !scales || !sums) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (k % 32u) return fail(EOS_E_INVALID_ARG, "k=%u is not a multiple of 32", k);
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {a, aq, scales, sums});
  if (rc != EOS_OK) return rc;
  if (m == 0 || k == 0) return EOS_OK;
  // Pack into a temporary source-order buffer, then scatter to the caller's arrays.
  const size_t bytes = eos::act_layout_bytes(m, k, EOS_ACT_LAYOUT_SOURCE);
  uint8_t* tmp = nullptr;
  EOS_CK(cudaMallocAsync(&tmp, bytes, (cudaStream_t)stream), "scratch");
  cudaError_t e = eos::launch_act_pack(a, m, k, tmp, EOS_ACT_LAYOUT_SOURCE, (cudaStream_t)stream);
  const size_t nq = (size_t)m * k, ng = (size_t)m * (k / 32u);
  if (e == cudaSuccess) e = cudaMemcpyAsync(aq, tmp, nq, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(scales, tmp + nq, ng * 4u, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(sums, tmp + nq + ng * 4u, ng * 4u, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  cudaFreeAsync(tmp, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "activation pack");
  return EOS_OK;
}

int eosi_cuda_unpack_scale_min_dev(const uint8_t* scales12, uint32_t count, uint8_t* sc, uint8_t* m,
                                   void* stream) {
  if (!scales12 || !sc || !m) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {scales12, sc, m});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_unpack_scale_min(scales12, count, sc, m, (cudaStream_t)stream), "unpack kernel");
  return EOS_OK;
}

int eosi_cuda_q8_0_quantize_dev(const float* src, void* dst, size_t n_elements, void* stream) {
  if (!src || !dst) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (n_elements % 32u) return fail(EOS_E_INVALID_ARG, "n_elements not a multiple of 32");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {src, dst});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_q80_quantize(src, (uint8_t*)dst, n_elements, (cudaStream_t)stream), "q8_0 quantize kernel");
  return EOS_OK;
}

int eosi_cuda_q4_k_quantize_dev(const float* src, void* dst, size_t n_elements, void* stream) {
  if (!src || !dst) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (n_elements % 256u) return fail(EOS_E_INVALID_ARG, "n_elements not a multiple of 256");
  if (!al16(dst)) return fail(EOS_E_INVALID_ARG, "dst must be 16-byte aligned");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {src, dst});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_q4k_quantize(src, (uint8_t*)dst, n_elements, (cudaStream_t)stream), "q4_k quantize kernel");
  return EOS_OK;
}

int eosi_cuda_fill_gauss_dev(float* dst, size_t n, uint64_t seed, uint64_t offset, float sigma, void* stream) {
  if (!dst) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {dst});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_fill_gauss(dst, n, seed, offset, sigma, (cudaStream_t)stream), "gauss kernel");
  return EOS_OK;
}

int eosi_cuda_q4_k_from_gauss_dev(void* dst, size_t n_elements, uint64_t seed, float sigma, void* stream) {
  if (!dst) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (n_elements % 256u) return fail(EOS_E_INVALID_ARG, "n_elements not a multiple of 256");
  if (!al16(dst)) return fail(EOS_E_INVALID_ARG, "dst must be 16-byte aligned");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info, {dst});
  if (rc != EOS_OK) return rc;
  EOS_CK(eos::launch_q4k_from_gauss((uint8_t*)dst, n_elements / 256u, seed, 0, sigma, (cudaStream_t)stream),
         "q4_k generator kernel");
  return EOS_OK;
}

int eosi_cuda_take_device_errors(uint32_t* bits) {
  if (!bits) return fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  DevInfo* info = nullptr;
  int rc = dev_prologue(&info);
  if (rc != EOS_OK) return rc;
  uint32_t v = 0;
  EOS_CK(cudaMemcpy(&v, info->err_d, 4, cudaMemcpyDeviceToHost), "read error word");
  if (v) EOS_CK(cudaMemset(info->err_d, 0, 4), "clear error word");
  uint32_t na = 0;  // and the no-alloc entry point's own word
  rc = eos::noalloc_take_errors(&na);
  if (rc != EOS_OK) return fail(rc, "read the no-alloc error word");
  *bits = v | na;
  return EOS_OK;
}

int eosi_cuda_set_kernel_variant(int b_dtype, int variant) {
  if (b_dtype == EOS_DT_Q4_K) {
    eos::set_q4k_gemv_variant(variant);
  } else if (b_dtype == EOS_DT_Q8_0) {
    eos::set_q80_gemv_variant(variant);
  } else {
    return fail(EOS_E_UNSUPPORTED, "dtype %d", b_dtype);
  }
  return EOS_OK;
}

}  // extern "C"
