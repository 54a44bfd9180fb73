// decoder_internal.h -- structures of the device-resident decoder
// (decoder.cu).  Internal: the public boundary is include/eosllm_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace eos {

// Words the step kernels share in device memory.
struct DecState {
  uint32_t pos;         // position of the next step == tokens consumed
  uint32_t n_prompt;    // steps at pos < n_prompt read their token from prompt[pos]
  uint32_t next_token;  // greedy pick of the previous step
  uint32_t arg_count;   // argmax CTA arrivals (reset by the last CTA)
  uint32_t err;         // EOS_DEVERR_* bits
  uint32_t epoch;       // completed steps (never reset): tensor-parallel exchange epochs
  uint32_t pad[2];
};

// Tensor-parallel receive words of one rank, in its exchange buffer; the
// other ranks write them through CUDA IPC mappings (push).  Flag values are
// epochs: step_epoch * (2 n_layer + 1) + exchange + 1.
struct XRecv {
  uint32_t flag[3][8];  // [0] O partial, [1] down partial, [2] argmax result; [.][q]: written by rank q
  float arg_v[8];       // rank q's best logit
  uint32_t arg_i[8];    // its global vocabulary index
  uint32_t first_nan;   // from rank 0: logits[0] is NaN
  uint32_t pad[7];
};

// One layer's resident weights (this rank's slices).
struct DecLayer {
  uint8_t* wqkv;  // [q rows; k rows; v rows] x n_embd
  uint8_t* wo;    // n_embd rows x (this rank's head columns)
  uint8_t* wgu;   // [gate rows; up rows] of this rank's FFN slice x n_embd
  uint8_t* wd;    // n_embd rows x (this rank's FFN columns)
  float* attn_norm;
  float* ffn_norm;
};

}  // namespace eos
