// eos_noalloc.cu -- a Q4_K matmul entry point that allocates no memory.
//
// Who needs it: hosts that must not allocate device memory once they are
// running.  Embedded and real-time deployments (the environments eosllm
// itself targets) commonly reserve every buffer at start-up and forbid
// allocation on the serving path, because cudaMalloc can block, can fail
// late under fragmentation, and breaks their memory budget; other hosts hand
// all device memory to their own pool allocator, so a library-side
// cudaMalloc would escape the pool's accounting.  eosi_cuda_matmul_q4_k_dev
// needs a caller-provided scratch buffer for the packed activations; this
// entry point instead uses one fixed array compiled into the library.
//
// The array is a file-scope __device__ variable of kNoAllocScratchBytes
// (1 MiB).  Every GPU that loads the library holds its own copy until the
// process exits.  Host code cannot use the array's name as a device address
// (on the host it only names a stand-in object), so the first call on each
// device looks the real address up with cudaGetSymbolAddress, with that
// device current, and passes it to the kernels.  A second file-scope word
// holds the device-side error bits of the most recent call on the device
// (zeroed by that call's packing kernel; a GEMV whose bounded wait ran out
// sets a bit): eosi_cuda_take_device_errors reports and clears it.
#include <mutex>

#include "eosllm_cuda.h"
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ uint32_t g_noalloc_err;

struct NoAllocDevice {
  bool ready = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  uint32_t* err = nullptr;     // device address of g_noalloc_err
  int num_sms = 0;
  int max_smem = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kMaxDevices];

// Set-up for the current device, done once: the scratch array's device
// address and the launch limits.  No allocation happens here either.
int noalloc_device(NoAllocDevice** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return EOS_E_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess || major != 10 ||
        minor != 0) {
      cudaGetLastError();
      return EOS_E_UNSUPPORTED;
    }
    void* ptr = nullptr;
    void* eptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr ||
        cudaGetSymbolAddress(&eptr, g_noalloc_err) != cudaSuccess || eptr == nullptr) {
      cudaGetLastError();
      return EOS_E_INTERNAL;
    }
    d.err = static_cast<uint32_t*>(eptr);
    if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
      cudaGetLastError();
      return EOS_E_INTERNAL;
    }
    d.scratch = static_cast<uint8_t*>(ptr);
    d.ready = true;
  }
  *out = &d;
  return EOS_OK;
}

int noalloc_fail(int status, const char* msg) {
  eos::set_error_message(msg);  // what eosi_cuda_last_error() returns
  return status;
}

}  // namespace

namespace eos {
// The error bits of the most recent no-alloc call on the current device, then
// cleared (0 when the device has made no such call).
int noalloc_take_errors(uint32_t* bits) {
  *bits = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return EOS_E_UNSUPPORTED;
  }
  uint32_t* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_dev[dev].ready) err = g_noalloc_dev[dev].err;
  }
  if (err == nullptr) return EOS_OK;
  uint32_t v = 0;
  if (cudaMemcpy(&v, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
      (v != 0 && cudaMemset(err, 0, 4) != cudaSuccess)) {
    cudaGetLastError();
    return EOS_E_INTERNAL;
  }
  *bits = v;
  return EOS_OK;
}
}  // namespace eos

extern "C" {

EOSLLM_CUDA_API int eosi_cuda_matmul_q4_k_noalloc(const float* a, const void* w, float* c, uint32_t m, uint32_t n,
                                                  uint32_t k, void* stream) {
  if (a == nullptr || w == nullptr || c == nullptr) return noalloc_fail(EOS_E_INVALID_ARG, "NULL pointer argument");
  if (k % Q4K_ELEMS) return noalloc_fail(EOS_E_INVALID_ARG, "q4_k: k is not a multiple of 256");
  if ((reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u))
    return noalloc_fail(EOS_E_INVALID_ARG, "device pointers must be 16-byte aligned");
  const size_t need = eos::act_layout_bytes(m, k, EOS_ACT_LAYOUT_GEMV);
  if (need > kNoAllocScratchBytes)
    return noalloc_fail(EOS_E_INVALID_ARG,
                        "q4_k no-alloc: m * k / 256 * 480 bytes of packed activations exceed the 1 MiB "
                        "built-in scratch (m * k must be <= 559104); use eosi_cuda_matmul_q4_k_dev");
  if (m == 0 || n == 0) return EOS_OK;
  NoAllocDevice* d = nullptr;
  const int rc = noalloc_device(&d);
  if (rc != EOS_OK) return noalloc_fail(rc, "no usable sm_100 device for the no-alloc entry point");
  int dev = 0;
  cudaGetDevice(&dev);
  if (eos::pointers_on_device({a, w, c}, dev) != EOS_OK) return EOS_E_INVALID_ARG;  // message already set
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n < 4) {  // the reference's f32-dequant path for n < 4 needs no scratch
    e = eos::launch_q4k_f32_small_n(a, static_cast<const uint8_t*>(w), c, m, n, k, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return noalloc_fail(EOS_E_INTERNAL, cudaGetErrorString(e));
    }
    return EOS_OK;
  }
  e = eos::launch_act_pack(a, m, k, d->scratch, EOS_ACT_LAYOUT_GEMV, st, d->err);
  const size_t stride = eos::act_layout_bytes(1, k, EOS_ACT_LAYOUT_GEMV);
  for (uint32_t i = 0; i < m && e == cudaSuccess; ++i) {
    int status = EOS_OK;
    e = eos::launch_q4k_gemv(static_cast<const uint8_t*>(w), d->scratch + i * stride, nullptr, c + (size_t)i * n, n,
                             k, d->err, d->num_sms, d->max_smem, true, st, &status);
    if (e == cudaSuccess && status != EOS_OK) return noalloc_fail(status, "q4_k gemv: shape not supported");
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return noalloc_fail(EOS_E_INTERNAL, cudaGetErrorString(e));
  }
  return EOS_OK;
}

}  // extern "C"
