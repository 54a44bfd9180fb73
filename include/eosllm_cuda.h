/*
 * eosllm_cuda.h -- C ABI of the B200 (sm_100a) backend for eosllm's
 * quantized matmul path (libeosllm_cuda.so).
 *
 * Plain C: no CUDA or C++ types in any signature.  Every function returns an
 * eos_status_t value as int (0 = EOS_OK, 1 = EOS_E_INVALID_ARG,
 * 2 = EOS_E_OUT_OF_MEMORY, 3 = EOS_E_UNSUPPORTED, 9 = EOS_E_INTERNAL;
 * include/eosllm/eosllm.h:66-77 of the reference), never aborts, and writes
 * outputs only on EOS_OK.  The last failure is described by
 * eosi_cuda_last_error().  Dtype codes are the reference's eos_dtype_t
 * (include/eosllm/tensor.h:32-33): 32 = Q8_0, 33 = Q4_K.
 *
 * Two layers:
 *   1. Host-pointer entry points with exactly the semantics of the
 *      reference's backend slot eos_backend_ops_t.matmul_q
 *      (include/eosllm/backend.h:43-46): synchronous, all pointers host
 *      memory owned by the caller, C = A . deq(B)^T row-major.  Weights are
 *      uploaded on first use and cached on the device(s), keyed by the host
 *      pointer, dtype and shape (plus a fingerprint of the first and last
 *      64 bytes, so a freed-and-reused address with new contents is
 *      re-uploaded).  Output rows are sharded across the configured GPUs.
 *   2. Device-pointer entry points (suffix _dev) that enqueue on a caller
 *      stream (a cudaStream_t passed as void*, NULL = legacy default stream)
 *      on the current device, for device-resident callers.
 */
#ifndef EOSLLM_CUDA_H
#define EOSLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EOSLLM_CUDA_API __attribute__((visibility("default")))
#else
#define EOSLLM_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- backend lifecycle ------------------------------------------------ */

/* EOS_OK when at least one sm_100 GPU is usable.  Cached after the first
 * call, so cheap enough for the registry to call at every session open.
 * Replaces the backend probe slot eos_backend_vt_t.probe
 * (include/eosllm/backend.h:71-76; cf. avx2_probe, src/kernels/avx2/avx2.c:79-81). */
EOSLLM_CUDA_API int eosi_cuda_probe(void);

/* Number of usable sm_100 devices (0 when none). */
EOSLLM_CUDA_API int eosi_cuda_device_count(void);

/* Select the GPUs the host-pointer entry points shard output rows across.
 * ids == NULL or count <= 0 restores the default: the list in the
 * EOSLLM_CUDA_DEVICES environment variable ("0,1,2"), else device 0.
 * Drops the weight cache. */
EOSLLM_CUDA_API int eosi_cuda_set_devices(const int *ids, int count);

/* Release every device buffer, stream and cached weight.  The next call
 * re-initialises lazily. */
EOSLLM_CUDA_API void eosi_cuda_shutdown(void);

/* Human-readable description of the last failure in this thread. */
EOSLLM_CUDA_API const char *eosi_cuda_last_error(void);

/* ---- host-pointer matmuls (the backend vtable slot) -------------------- */

/* eos_backend_ops_t.matmul_q replacement (include/eosllm/backend.h:43-46);
 * dispatch as in eosi_avx2_matmul_q (src/kernels/avx2/matmul_q4_k.c:155-171):
 * Q4_K and Q8_0 run on the GPU, any other dtype is EOS_E_UNSUPPORTED. */
EOSLLM_CUDA_API int eosi_cuda_matmul_q(const float *a, const void *b_quant, int b_dtype, float *c,
                       uint32_t m, uint32_t n, uint32_t k);

/* Q4_K: replaces eosi_avx2_matmul_q4_k_int8
 * (src/kernels/avx2/matmul_q4_k_int8.c:164-269) and is bit-identical to it:
 * activations packed to int8 exactly as quantize_sub32 (:98-154), exact
 * integer sub-block dots, fp32 rescale in the reference's order.  k % 256
 * must be 0 (EOS_E_INVALID_ARG otherwise, as at :173-174).  For n < 4 the
 * reference routes to its f32-dequant path eosi_avx2_matmul_q4_k (:182-184,
 * src/kernels/avx2/matmul_q4_k.c:70-153); so does this backend, with the
 * same eight FMA accumulator lanes and horizontal sum, again bit-identical. */
EOSLLM_CUDA_API int eosi_cuda_matmul_q4_k(const float *a, const void *b_q4, float *c,
                          uint32_t m, uint32_t n, uint32_t k);

/* Q8_0: replaces eosi_scalar_matmul_q8_0 (src/kernels/scalar/matmul_q8.c:21-58),
 * f32 activations; agrees to fp32 rounding (different summation order).
 * k % 32 must be 0. */
EOSLLM_CUDA_API int eosi_cuda_matmul_q8_0(const float *a, const void *b_q8, float *c,
                          uint32_t m, uint32_t n, uint32_t k);

/* Forget the cached device copy of one host weight buffer (or of all). */
EOSLLM_CUDA_API int eosi_cuda_cache_evict(const void *b_quant);
EOSLLM_CUDA_API int eosi_cuda_cache_clear(void);

/* Counters of the host-pointer path (reading them launches nothing): the matmuls completed on
 * the GPU through eosi_cuda_matmul_q / _q4_k / _q8_0 since the library was
 * loaded, and the weight-cache entries (one per weight and device) with their
 * device bytes.  An engine integration reads them to confirm that its
 * dispatch really routes matmul_q here.  NULL arguments are skipped. */
EOSLLM_CUDA_API int eosi_cuda_host_stats(uint64_t *calls, uint64_t *cached_weights, uint64_t *cached_bytes);

/* Upload (or refresh) one weight buffer now instead of on first use. */
EOSLLM_CUDA_API int eosi_cuda_cache_preload(const void *b_quant, int b_dtype, uint32_t n, uint32_t k);

/* ---- device-pointer entry points (current device, caller stream) ------- */

/* Scratch the Q4_K entry points need for m activation rows of length k:
 * the packed int8 activations, scales and sums (480 bytes per 256 of k). */
EOSLLM_CUDA_API size_t eosi_cuda_q4_k_scratch_bytes(uint32_t m, uint32_t k);

/* C[m,n] = A[m,k] . deq(W)^T with A, W, C and scratch in device memory.
 * W is n rows of k/256 GGUF Q4_K super-blocks, 16-byte aligned; A and
 * scratch 16-byte aligned; scratch >= eosi_cuda_q4_k_scratch_bytes(m, k).
 * With scratch, activations are packed by a separate kernel chained to the
 * GEMV (programmatic dependent launch).  For m == 1 scratch may be NULL:
 * every CTA of the GEMV then packs the vector itself into shared memory
 * (rows too long to stage in shared memory still need scratch).
 * Asynchronous on `stream`; bit-identical to eosi_cuda_matmul_q4_k. */
EOSLLM_CUDA_API int eosi_cuda_matmul_q4_k_dev(const float *a, const void *w, float *c, uint32_t m, uint32_t n,
                              uint32_t k, void *scratch, void *stream);

/* The two halves of eosi_cuda_matmul_q4_k_dev, for callers that pack one
 * activation vector once and multiply it by several weights:
 *   pack: a[m,k] -> act (eosi_cuda_q4_k_scratch_bytes(m, k) bytes);
 *   gemv: c[n] = act(row 0) . deq(W)^T. */
EOSLLM_CUDA_API int eosi_cuda_q4_k_pack_act_dev(const float *a, uint32_t m, uint32_t k, void *act, void *stream);
EOSLLM_CUDA_API int eosi_cuda_q4_k_gemv_dev(const void *act, const void *w, float *c, uint32_t n, uint32_t k,
                            void *stream);

/* Q4_K matmul that allocates nothing -- no counterpart in the reference.
 * For hosts that may not allocate device memory while running (all buffers
 * reserved at start-up, or all device memory owned by the host's own pool):
 * the same computation as eosi_cuda_matmul_q4_k_dev, bit-identical results,
 * but the packed activations live in a 1 MiB array built into the library
 * instead of a caller scratch buffer.  Limits and behaviour:
 *   - m * k / 256 * 480 bytes must fit in 1 MiB (m * k <= 559104, e.g. one
 *     row of k up to 559104, or m <= 136 rows of k = 4096); larger sizes
 *     return EOS_E_INVALID_ARG with a message;
 *   - each GPU that loads the library keeps its own copy of the array until
 *     the process exits;
 *   - the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture;
 *   - every call on a device reuses the same array, so calls whose work
 *     overlaps on that GPU (other streams, other host threads) race and
 *     corrupt each other's results -- serialise them;
 *   - no cudaMalloc, cudaFree or other allocating call is made;
 *   - the GEMV's waits for its staged weights are bounded: one that runs out
 *     sets a bit in the entry point's own error word (also in the library's
 *     image, started at 0 by each call), which eosi_cuda_take_device_errors
 *     reports after the stream has been synchronised;
 *   - under CUDA's default lazy module loading the driver itself loads each
 *     kernel on its first launch, and loading takes device memory: a host
 *     that must see no allocation on its serving path makes one warm-up
 *     call per (m, n, k) shape class it will use at start-up (n < 4, k whose
 *     packed row fits in shared memory, longer k) or runs with
 *     CUDA_MODULE_LOADING=EAGER.
 * a, w, c are device pointers on the current device (a and w 16-byte
 * aligned); `stream` is a cudaStream_t as void*; asynchronous. */
EOSLLM_CUDA_API int eosi_cuda_matmul_q4_k_noalloc(const float *a, const void *w, float *c, uint32_t m, uint32_t n,
                                                  uint32_t k, void *stream);

/* Q8_0 with device pointers (W 16-byte aligned, k % 256 == 0 on this path). */
EOSLLM_CUDA_API int eosi_cuda_matmul_q8_0_dev(const float *a, const void *w, float *c, uint32_t m, uint32_t n,
                              uint32_t k, void *stream);

/* Activation packing in source order, for checking it against
 * quantize_sub32 (src/kernels/avx2/matmul_q4_k_int8.c:98-154) bit for bit:
 * aq[m*k] int8, scales[m*k/32] f32, sums[m*k/32] int32. */
EOSLLM_CUDA_API int eosi_cuda_quantize_act_dev(const float *a, uint32_t m, uint32_t k, int8_t *aq, float *scales,
                               int32_t *sums, void *stream);

/* Scale/min unpack of `count` 12-byte Q4_K scale fields into 8 sc and 8 m
 * bytes each -- the GEMV's own unpack, checked against get_scale_min
 * (src/kernels/avx2/matmul_q4_k_int8.c:58-67). */
EOSLLM_CUDA_API int eosi_cuda_unpack_scale_min_dev(const uint8_t *scales12, uint32_t count, uint8_t *sc, uint8_t *m,
                                   void *stream);

/* ---- weight formats and synthetic data on the device ------------------- */

/* Q8_0 weight quantizer: src/quant/q8_0.c:58-93, bit for bit. */
EOSLLM_CUDA_API int eosi_cuda_q8_0_quantize_dev(const float *src, void *dst, size_t n_elements, void *stream);

/* Q4_K weight quantizer.  The reference has none (src/quant/q4_k.c:83-93
 * returns EOS_E_UNSUPPORTED); this is the project's affine min/max fit,
 * dequantized by the reference's q4_k_dequantize (src/quant/q4_k.c:42-81). */
EOSLLM_CUDA_API int eosi_cuda_q4_k_quantize_dev(const float *src, void *dst, size_t n_elements, void *stream);

/* Seeded synthetic values (Irwin-Hall(12) normal approximation on
 * splitmix64; element i of stream `seed` is identical on host and device). */
EOSLLM_CUDA_API int eosi_cuda_fill_gauss_dev(float *dst, size_t n, uint64_t seed, uint64_t offset, float sigma,
                             void *stream);

/* Generator fused into the Q4_K quantizer: n_elements synthetic values of
 * stream `seed` (offset 0) quantized straight to Q4_K without an f32 copy. */
EOSLLM_CUDA_API int eosi_cuda_q4_k_from_gauss_dev(void *dst, size_t n_elements, uint64_t seed, float sigma,
                                  void *stream);

/* ---- tensor-core prefill (m > 1) ----------------------------------------------
 * C[m,n] = A[m,k] . deq(W)[n,k]^T on the sm_100a tensor cores (tcgen05),
 * bit-exact with eosi_cuda_matmul_q4_k and with the reference's int8 kernel
 * (src/kernels/avx2/matmul_q4_k_int8.c:164-269), which the reference applies
 * to one prompt token at a time (src/core/session.c:231-236).  Activations
 * are packed per 32 exactly as quantize_sub32 does (the int8 values held as
 * bf16, which is exact); every sub-block's integer dot is two bf16 x bf16
 * tensor-core MMAs (tcgen05 kind::f16, K = 16 each) into an f32 TMEM
 * accumulator -- exact, since every product and partial sum is an integer
 * below 2^16 -- then rescaled and summed in the reference's f32 order.
 * Weights are prepared once into eosi_cuda_q4_k_prefill_weight_bytes bytes
 * (the 4-bit values as bf16 plus per-32 (d*sc, -(dmin*m)) pairs); each call
 * needs eosi_cuda_q4_k_prefill_scratch_bytes of scratch.  All pointers device,
 * 16-byte aligned; k % 256 == 0. */
EOSLLM_CUDA_API size_t eosi_cuda_q4_k_prefill_weight_bytes(uint32_t n, uint32_t k);
EOSLLM_CUDA_API size_t eosi_cuda_q4_k_prefill_scratch_bytes(uint32_t m, uint32_t k);
EOSLLM_CUDA_API int eosi_cuda_q4_k_prefill_prepare_weights_dev(const void *w, uint32_t n, uint32_t k, void *w_prep,
                                                               void *stream);
EOSLLM_CUDA_API int eosi_cuda_q4_k_prefill_dev(const float *a, const void *w_prep, float *c, uint32_t m, uint32_t n,
                                               uint32_t k, void *scratch, void *stream);

/* ---- device-resident Llama decoder ------------------------------------------
 * The work of eosi_text_open / eosi_text_step / eosi_text_close
 * (src/modality/text/text.h:62-78, text.c:131-436 of the reference) with
 * every weight, the KV cache and the greedy pick (src/sched/greedy.c:48-73)
 * on one GPU, or row/column-sharded across `world` GPUs (one process per
 * GPU, rank r on its own device).  Linears are Q4_K or Q8_0, token
 * embeddings F16, norms F32, the KV cache f32 like the reference's. */
typedef struct {
    uint32_t n_embd, n_layer, n_head, n_kv_head, n_ff, n_vocab, max_ctx;
    float rms_eps, rope_base;
    int32_t wdtype;            /* 33 (Q4_K) or 32 (Q8_0): every block linear */
    int32_t out_dtype;         /* dtype of output.weight */
    int32_t weights_on_device; /* 0: host pointers (e.g. into the GGUF buffer);
                                  1: device pointers on `device` */
    const uint16_t *tok_embd;  /* F16 [n_vocab][n_embd] */
    const float *output_norm;  /* F32 [n_embd] */
    const void *output_w;      /* [n_vocab] rows of n_embd */
    /* per-layer tables of n_layer pointers, GGUF row-major (one row per
     * output): attn_q [n_embd], attn_k / attn_v [n_kv_head*head_dim],
     * attn_output [n_embd], ffn_gate / ffn_up [n_ff] rows of n_embd,
     * ffn_down [n_embd] rows of n_ff */
    const float *const *attn_norm;
    const float *const *ffn_norm;
    const void *const *wq;
    const void *const *wk;
    const void *const *wv;
    const void *const *wo;
    const void *const *wg;
    const void *const *wu;
    const void *const *wd;
} eosi_cuda_llama_t;

typedef struct eosi_cuda_text eosi_cuda_text_t;

/* Upload this rank's slices of the model to `device` and build the per-token
 * step.  head_dim must be 64, 128 or 256; n_embd a multiple of 256; `world`
 * must divide n_head and n_kv_head.  Replaces eosi_text_open (text.c:131-260). */
EOSLLM_CUDA_API int eosi_cuda_text_open(const eosi_cuda_llama_t *m, int device, int rank, int world,
                                        eosi_cuda_text_t **out);
/* How a step runs.  PER_OP: a CUDA graph of one kernel per operation,
 * chained with programmatic dependent launch (any supported model).
 * PERSISTENT: one cooperative kernel per token, one CTA per SM, every weight
 * matrix streamed through per-warp TMA rings that run ahead across the
 * step's phases, every vector that crosses CTAs or ranks as (epoch, word)
 * pairs (Q4_K linears and LM head, head_dim 64 or 128, n_embd <= 4096).  Both
 * give bit-identical logits and tokens.  AUTO (the default) is PER_OP, the
 * faster of the two on a B200 for the 7B shape (about 695 against 470
 * tokens/s).  Tensor parallel: every rank sets the same mode, with no step
 * running.  EOS_E_UNSUPPORTED when PERSISTENT is asked for and not
 * possible. */
#define EOSI_CUDA_STEP_AUTO 0
#define EOSI_CUDA_STEP_PERSISTENT 1
#define EOSI_CUDA_STEP_PER_OP 2
EOSLLM_CUDA_API int eosi_cuda_text_set_step_mode(eosi_cuda_text_t *t, int mode);
/* The mode in use: EOSI_CUDA_STEP_PERSISTENT or EOSI_CUDA_STEP_PER_OP. */
EOSLLM_CUDA_API int eosi_cuda_text_step_mode(const eosi_cuda_text_t *t);
/* One decoder step at the current position: token -> logits[n_vocab]
 * (host memory), position + 1.  Same contract as eosi_text_step
 * (text.c:267-436): EOS_E_INVALID_ARG for token >= n_vocab,
 * EOS_E_OUT_OF_MEMORY when the context is full. */
EOSLLM_CUDA_API int eosi_cuda_text_step(eosi_cuda_text_t *t, uint32_t token, float *logits);
/* Greedy generation without a host round trip per token: feeds prompt
 * [0, n_prompt) from the current position, then n_gen - 1 of its own picks,
 * and returns the n_gen picks (the first is the pick after the last prompt
 * token), as eos_session_feed + eos_session_step with the greedy scheduler
 * do (src/core/session.c:211-262, src/sched/greedy.c:48-73). */
EOSLLM_CUDA_API int eosi_cuda_text_generate(eosi_cuda_text_t *t, const uint32_t *prompt, uint32_t n_prompt,
                                            uint32_t n_gen, uint32_t *out_tokens);
/* Batched prefill: feeds tokens[0, n) from the current position in one pass
 * per layer on the tensor cores (the KV cache rows of all n tokens), with no
 * logits; position + n.  The reference feeds a prompt token by token
 * (src/core/session.c:231-236); the linears here are bit-exact with it and
 * the cache rows differ only by the attention sums' rounding.  Q4_K linears only, else EOS_E_UNSUPPORTED (feed the
 * tokens with eosi_cuda_text_step instead); tensor parallel, every rank
 * makes the same call (the partial sums are exchanged like the step's).
 * eosi_cuda_text_generate uses it for all prompt tokens but the last when at
 * least `min_tokens` precede the last (eosi_cuda_text_set_prefill_min; default
 * 16, 0 = never). */
EOSLLM_CUDA_API int eosi_cuda_text_prefill(eosi_cuda_text_t *t, const uint32_t *tokens, uint32_t n);
EOSLLM_CUDA_API int eosi_cuda_text_set_prefill_min(eosi_cuda_text_t *t, uint32_t min_tokens);
/* The batched prefill's linears read weights prepared into the tensor-core
 * layout (4-bit values as bf16 plus per-32 scales, 2.25 bytes per weight).
 * resident != 0 (default): all layers are prepared once, at the first
 * prefill, when that fits in half of the free device memory, and kept;
 * 0: each matrix is prepared into a scratch buffer just before its GEMM. */
EOSLLM_CUDA_API int eosi_cuda_text_set_prefill_resident(eosi_cuda_text_t *t, int resident);
/* Position back to 0 (the KV cache is overwritten as steps proceed). */
EOSLLM_CUDA_API int eosi_cuda_text_reset(eosi_cuda_text_t *t);
EOSLLM_CUDA_API uint32_t eosi_cuda_text_pos(const eosi_cuda_text_t *t);
/* Tensor parallel (world > 1): after eosi_cuda_text_open on every rank, each
 * rank exports the IPC handle of its exchange buffer (EOSI_CUDA_IPC_HANDLE_BYTES
 * bytes), the host gathers all ranks' handles in rank order (e.g. an
 * all-gather over the process group) and passes them to
 * eosi_cuda_text_attach_peers, which maps the peers' buffers and builds the
 * step.  Every matrix is split by output rows (the q/k/v rows of a rank's
 * heads, the gate/up rows of its FFN units, a slice of the O and down output
 * rows, a slice of the vocabulary), so every output element is computed
 * whole on one rank, exactly as on one GPU.  Per layer the ranks exchange,
 * by pushing into each other's buffers over NVLink, the attention output
 * (packed for the O projection), the O output rows, the SiLU output (packed
 * for the down projection) and the down output rows, and at the end their
 * slice's greedy pick; every rank therefore holds the one-GPU residual
 * stream bit for bit and picks the one-GPU tokens.  Every word pushed
 * carries its exchange's epoch in the same 64-bit store, so a consumer polls
 * the words themselves in its own memory; the pick is a flag handshake.
 * Every wait is bounded (one second unless eosi_cuda_text_set_wait_limit
 * says otherwise; EOS_E_INTERNAL when a rank never arrives).  Every rank must make the same calls in the same order
 * (step / generate / prefill / reset). */
#define EOSI_CUDA_IPC_HANDLE_BYTES 64
EOSLLM_CUDA_API int eosi_cuda_text_ipc_handle(eosi_cuda_text_t *t, void *out, size_t cap);
EOSLLM_CUDA_API int eosi_cuda_text_attach_peers(eosi_cuda_text_t *t, const void *handles, size_t bytes);
/* The same attachment for ranks opened in ONE process (one host thread
 * driving every rank; ranks on different devices get peer access enabled):
 * ranks[q] is rank q's decoder.  Every rank must then be stepped; a rank
 * that is not makes the others' next exchange run into its bounded wait. */
EOSLLM_CUDA_API int eosi_cuda_text_attach_local(eosi_cuda_text_t *const *ranks, int world);
/* Bound on every wait of this decoder's steps (tensor-parallel exchanges, and
 * the persistent step's waits for other CTAs' outputs), in microseconds
 * (default 1000000). */
EOSLLM_CUDA_API int eosi_cuda_text_set_wait_limit(eosi_cuda_text_t *t, uint32_t limit_us);
/* This rank's slice of the model (host only, no GPU needed): out[11] =
 * {head_dim, head0, heads, kv_head0, kv_heads, ff0, ff_len, vocab0,
 * vocab_len, out_row0, out_rows} (out_row*: the O / down output rows). */
EOSLLM_CUDA_API int eosi_cuda_text_partition(const eosi_cuda_llama_t *m, int rank, int world, uint32_t *out);
/* The decoder's cudaStream_t (as void*), for timing with events. */
/* Kernels one step launches (the nodes of its CUDA graph; 0 before the
 * step is built). */
EOSLLM_CUDA_API uint32_t eosi_cuda_text_step_kernels(const eosi_cuda_text_t *t);
EOSLLM_CUDA_API void *eosi_cuda_text_stream(eosi_cuda_text_t *t);
EOSLLM_CUDA_API void eosi_cuda_text_close(eosi_cuda_text_t *t);

/* ---- GGUF straight to the device -------------------------------------------
 * eosi_cuda_gguf_map parses a GGUF v3 Llama-family file with the reference's
 * rules (src/format/gguf/gguf.c; keys and tensors as eosi_text_open reads
 * them, src/modality/text/text.c:104-215) from a read-only memory mapping,
 * without reading it into host memory, and fills `desc` with pointers into
 * the mapping (valid until eosi_cuda_gguf_unmap); no GPU is needed.  Errors
 * as the reference's: EOS_E_IO (cannot open / map), EOS_E_FORMAT (bad magic,
 * version, truncation, shapes, missing tensors), EOS_E_NOT_FOUND (a required
 * key), EOS_E_UNSUPPORTED (tensor types the decoder cannot run: non-F16
 * embeddings, a tied output, mixed linear types).  max_ctx: 0 keeps the
 * file's context_length, else min(context_length, max_ctx).
 * eosi_cuda_text_open_gguf = map + eosi_cuda_text_open + unmap: each rank
 * copies only its own slices from the file to its GPU. */
typedef struct eosi_cuda_gguf eosi_cuda_gguf_t;
EOSLLM_CUDA_API int eosi_cuda_gguf_map(const char *path, uint32_t max_ctx, eosi_cuda_gguf_t **out,
                                       eosi_cuda_llama_t *desc);
EOSLLM_CUDA_API void eosi_cuda_gguf_unmap(eosi_cuda_gguf_t *g);
EOSLLM_CUDA_API int eosi_cuda_text_open_gguf(const char *path, uint32_t max_ctx, int device, int rank, int world,
                                             eosi_cuda_text_t **out);

/* ---- diagnostics --------------------------------------------------------- */

/* Device-side error bits raised by bounded waits since the last call on the
 * current device (0 = none), together with those of the most recent
 * eosi_cuda_matmul_q4_k_noalloc call on it (its own word, in the library's
 * image: each such call starts it at 0); clears them. */
EOSLLM_CUDA_API int eosi_cuda_take_device_errors(uint32_t *bits);

/* Kernel variant override for tuning (-1 = automatic).  Q4_K GEMV:
 * variant = config + 32 * rows_per_stage + 512 * ctas_per_sm + 4096 * chunk,
 * every field 0 = automatic; configs 0..11 are the row-major kernel (rows per
 * stage 1, 2, 4 or 8), 12..19 the column-major one, whose rows are staged
 * whole (chunk 1) or in pieces of 8 * (chunk - 1) super-blocks (chunk >= 2).
 * Every variant gives bit-identical results. */
EOSLLM_CUDA_API int eosi_cuda_set_kernel_variant(int b_dtype, int variant);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* EOSLLM_CUDA_H */
