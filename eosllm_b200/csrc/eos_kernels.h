// eos_kernels.h -- internal launch interface between the C-ABI layer
// (eos_backend.cu) and the kernel files.  Not installed; the public
// boundary is include/eosllm_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <initializer_list>

namespace eos {
struct LLExchange;  // eos_common.cuh
}

// Layouts the activation packer can write.
enum { EOS_ACT_LAYOUT_GEMV = 0, EOS_ACT_LAYOUT_SOURCE = 1 };

namespace eos {

// Sets the calling thread's message returned by eosi_cuda_last_error().
void set_error_message(const char* msg);
// EOS_OK when every non-null pointer is device (or managed) memory of device
// `dev`; else EOS_E_INVALID_ARG with the message set.  No allocation.
int pointers_on_device(std::initializer_list<const void*> ptrs, int dev);

size_t act_layout_bytes(uint32_t m, uint32_t k, int layout);
// zero_word (optional): set to 0 by the kernel, for the GEMVs that follow to
// report into (the host path reads it back with their outputs).
cudaError_t launch_act_pack(const float* a, uint32_t m, uint32_t k, uint8_t* out, int layout, cudaStream_t st,
                            uint32_t* zero_word = nullptr);

// Exactly one of `act` (packed activations, GEMV layout) and `a` (f32
// activations, packed inside the kernel) is non-null.  out_status: EOS_OK, or
// EOS_E_UNSUPPORTED when the shape cannot be staged on the fused path (the
// caller then packs separately).
// c_extra / n_extra (<= 7): further destinations of every output, written
// after c (tensor-parallel push into other GPUs' IPC-mapped buffers; visible
// to them once the grid has completed); not supported by the unstaged
// fallback.
// ll (optional, ll->epoch_word != nullptr): tensor parallel -- the packed
// activation records are read as the (epoch, word) pairs every rank pushed
// into ll->in (polled, bounded), and every output r goes as a pair to
// ll->out[j] + r instead of to c (see LLExchange).
cudaError_t launch_q4k_gemv(const uint8_t* w, const uint8_t* act, const float* a, float* c, uint32_t n, uint32_t k,
                            uint32_t* err, int num_sms, int max_smem, bool pdl, cudaStream_t st, int* out_status,
                            float* const* c_extra = nullptr, uint32_t n_extra = 0, const LLExchange* ll = nullptr);
void set_q4k_gemv_variant(int v);
// The device error bits of the most recent eosi_cuda_matmul_q4_k_noalloc call
// on the current device, then cleared (eos_noalloc.cu).
int noalloc_take_errors(uint32_t* bits);
// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// device memory written by the previous kernel on `st` to `dst`, typically
// the device alias of mapped pinned host memory.  Launched with programmatic
// dependent launch, so it replaces a device-to-host copy-engine transfer
// behind that kernel without waiting for a copy engine.
cudaError_t launch_copy_out(const void* src, void* dst, size_t bytes, cudaStream_t st);
// A one-thread kernel that sets *flag = 1 (device alias of mapped host
// memory) after the stream's earlier kernels.
cudaError_t launch_done_flag(uint32_t* flag, cudaStream_t st);
// n < 4 Q4_K: the reference's f32-dequant path, bit for bit.
cudaError_t launch_q4k_f32_small_n(const float* a, const uint8_t* w, float* c, uint32_t m, uint32_t n, uint32_t k,
                                   cudaStream_t st);

// Tensor-core prefill (prefill_gemm.cu), bit-exact with the int8 reference.
// Operand buffers: int8 values [rows][k], then at align1024(rows*k) the
// per-32 scale pairs [k/32][pad4(rows)]; prefill_operand_bytes gives the size.
size_t prefill_operand_bytes(uint32_t rows, uint32_t k);
cudaError_t launch_prefill_act_pack(const float* a, uint32_t m, uint32_t k, void* act, cudaStream_t st);
cudaError_t launch_prefill_w_prep(const uint8_t* w, uint32_t n, uint32_t k, void* wprep, cudaStream_t st);
// accumulate: C = C_old + A.W^T (the decoder's residual adds).  c_extra /
// n_extra (<= 7, not with accumulate): further destinations of C (tensor-
// parallel push into other GPUs' IPC-mapped buffers).  ldc: floats between
// rows of C and of every extra destination (0: n).
cudaError_t launch_prefill_gemm(const void* act, const void* wprep, float* c, uint32_t m, uint32_t n, uint32_t k,
                                uint32_t* err, cudaStream_t st, int* out_status, bool accumulate = false,
                                float* const* c_extra = nullptr, uint32_t n_extra = 0, uint32_t ldc = 0);

cudaError_t launch_q80_gemv(const uint8_t* w, const float* a, float* c, uint32_t n, uint32_t k, uint32_t* err,
                            int num_sms, int max_smem, cudaStream_t st, int* out_status,
                            float* const* c_extra = nullptr, uint32_t n_extra = 0, const LLExchange* ll = nullptr);
void set_q80_gemv_variant(int v);

// Test/utility kernels (eos_util.cu).
cudaError_t launch_unpack_scale_min(const uint8_t* scales12, uint32_t count, uint8_t* sc, uint8_t* m,
                                    cudaStream_t st);
cudaError_t launch_fill_gauss(float* dst, size_t n, uint64_t seed, uint64_t offset, float sigma, cudaStream_t st);
cudaError_t launch_q4k_quantize(const float* src, uint8_t* dst, size_t n_el, cudaStream_t st);
cudaError_t launch_q80_quantize(const float* src, uint8_t* dst, size_t n_el, cudaStream_t st);
// Generator fused into the Q4_K quantizer: super-block b quantizes the
// generated elements offset + 256b .. offset + 256b + 255.
cudaError_t launch_q4k_from_gauss(uint8_t* dst, size_t nblocks, uint64_t seed, uint64_t offset, float sigma,
                                  cudaStream_t st);

}  // namespace eos
