/* qwen_b200.h — C ABI of the B200 (sm_100a) Qwen3-0.6B batch-1 decode engine.
 *
 * Plain C: pointers, sizes and status codes only; no C++ or torch types.
 * Every entry point returns QWEN_OK (0) or a negative status; qwen_last_error()
 * gives the message of the last failure on the calling thread.  Nothing here
 * calls exit().  A handle owns all of its device memory and one CUDA stream on
 * one device; it is not thread-safe (one handle per GPU, one host thread each).
 *
 * Each declaration names the reference interface it replaces
 * (Ramshankar07/qwen600-ROCm-inference, file:line).
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QWEN_OK             0
#define QWEN_E_ARG         -1   /* bad argument: token/pos out of range, NULL pointer, bad shape */
#define QWEN_E_IO          -2   /* cannot open / read / map the checkpoint */
#define QWEN_E_FORMAT      -3   /* checkpoint header or tensor table does not match the model */
#define QWEN_E_CUDA        -4   /* a CUDA runtime call failed */
#define QWEN_E_TIMEOUT     -5   /* a bounded device-side wait ran out; device state was reset */
#define QWEN_E_UNSUPPORTED -6   /* valid request this build does not serve (e.g. top_k > 64 on device) */
#define QWEN_E_STATE       -7   /* call out of order (e.g. pos not contiguous with the cache) */

typedef struct qwen_ctx qwen_t;

/* Sampling parameters of sampler.h's Sampler (sampler.h:17-24, 99-112).
 * temperature == 0 or top_k == 1 selects argmax (sampler.h:125-128);
 * top_k == 0 means the whole vocabulary (sampler.h:109);
 * topp outside (0, 1) disables the nucleus cut (sampler.h:153). */
typedef struct {
    float temperature;
    float topp;
    int   top_k;
} qwen_sampling_t;

/* Message of the last error on this thread ("" if none). */
const char* qwen_last_error(void);

/* ABI version (major*10000 + minor*100 + patch). */
int qwen_abi_version(void);

/* ---- checkpoint (static_loader.h) --------------------------------------- */

/* Number of tensors in the model's canonical weight layout (static_loader.h:81, NUM_TENSORS = 311). */
int qwen_num_tensors(void);

/* VOCAB_SIZE of this build (config.h); lets callers size logits buffers without
 * config.h.  No reference counterpart (the reference uses the constant). */
int qwen_vocab_size(void);

/* Total bytes of the canonical device weight block (static_loader.h:80, TOTAL_WEIGHTS_BYTES). */
size_t qwen_total_weight_bytes(void);

/* Entry i of the canonical table: name, byte offset from the block start, size in bytes
 * (static_loader.h:83-400, TENSOR_METADATA).  The offsets are the order-sorted
 * safetensors layout of Qwen3-0.6B; the table is derived, not stored. */
int qwen_tensor_info(int index, const char** name, size_t* offset, size_t* bytes);

/* Parse and validate a safetensors checkpoint on the host only (no GPU needed):
 * the JSON header, every tensor's dtype/shape, and the file size.  The tensors
 * may appear in any order.  Replaces the header read of static_loader.h:415-427. */
int qwen_checkpoint_validate(const char* path);

/* Write the reference's ordered weight blob (weights_qwen600.bin, export.py:80-146)
 * of a BF16 safetensors checkpoint: the raw tensors back to back, no header, in
 * the order embed_tokens, lm_head, final norm, then per layer q, k, v, o,
 * q_norm, k_norm, gate, up, down, input_layernorm, post_attention_layernorm.
 * Every loading entry point (qwen_create, qwen_weights_load,
 * qwen_checkpoint_validate) accepts such a blob in place of the safetensors
 * file, and, like static_loader.hip.h:185-202, reads weights_qwen600.bin from
 * the checkpoint's directory instead of the checkpoint when one of the exact
 * size lies there. */
int qwen_write_ordered_blob(const char* safetensors_path, const char* out_path);

/* Load a checkpoint into ONE device allocation laid out in the canonical order
 * (static_loader.h:402-494, load_qwen_weights).  *dev_block receives the device
 * pointer (free with qwen_weights_free); tensor i sits at qwen_tensor_info(i).offset. */
int qwen_weights_load(const char* path, int device, void** dev_block);
int qwen_weights_free(void* dev_block);

/* Write a synthetic Qwen3-0.6B checkpoint (valid safetensors, canonical layout):
 * every matrix ~ N(0, 0.02) rounded to bf16 from a counter-based generator keyed
 * by `seed`, every RMSNorm / QK-norm gain 1.0, lm_head.weight == embed_tokens.weight.
 * Stands in for the exporter's weights (export.py:39-146) where no real
 * checkpoint is available. */
int qwen_write_synthetic_checkpoint(const char* path, uint64_t seed);

/* ---- model (qwen_model.cuh) --------------------------------------------- */

/* Load weights, allocate the KV cache and work buffers on `device`
 * (qwen_model.cuh:82-92, build_transformer). */
int qwen_create(const char* safetensors_path, int device, qwen_t** out);

/* Free everything the handle owns (qwen_model.cuh:94-111, free_transformer). */
void qwen_destroy(qwen_t* ctx);

/* Device the handle lives on. */
int qwen_device(const qwen_t* ctx);

/* One position of the decode chain (qwen_model.cuh:772-851, forward): embeds
 * `token`, appends its K/V at `pos` and computes the VOCAB_SIZE fp32 logits.
 * Positions must arrive in order 0..pos (pos <= the number of cached
 * positions).  If logits_host is non-NULL the logits are copied there before
 * return (the reference's blocking D2H, qwen_model.cuh:848). */
int qwen_forward(qwen_t* ctx, int token, int pos, float* logits_host);

/* Pinned host buffer of VOCAB_SIZE floats owned by the handle (qwen_model.cuh:59,
 * Transformer.h_logits); qwen_forward(ctx, t, p, qwen_host_logits(ctx)) is the
 * reference's forward() contract. */
float* qwen_host_logits(qwen_t* ctx);

/* Device pointer to the fp32 logits of the last forward / decode step. */
const float* qwen_device_logits(qwen_t* ctx);

/* Device pointer to the handle's weight block, in the canonical layout of
 * qwen_tensor_info (tensor i at offset i); the handle owns it.  Lets the C++
 * names fill Transformer.weights (qwen_model.cuh:53, TransformerWeights
 * weights) with pointers a reference-written caller can index. */
const void* qwen_device_weights(const qwen_t* ctx);

/* Copy the fp32 logits of the last forward / decode / generate step (the rows
 * this handle serves: all VOCAB_SIZE, or its vocabulary shard) to host memory;
 * returns the number of floats copied.  The reference's forward() hands these
 * back every call (qwen_model.cuh:848); here the copy is on request. */
int qwen_read_logits(qwen_t* ctx, float* logits_host);

/* forward(token, pos) followed by sample() on the device (main.cu:144-145 with
 * sampler.h:120-175): *next_token receives the sampled id and *rng_state the
 * advanced xorshift64* state.  Only 4 + 8 bytes come back to the host.
 * The device samples argmax and, with the nucleus cut on (0 < topp < 1),
 * 1 <= top_k <= 64 candidates.  Every other setting (topp outside (0, 1),
 * top_k = 0 or > 64) draws on the host from the step's device logits with
 * qwen_sample_host, because the reference's candidate order is then the
 * partition order of its quickselect over the whole vocabulary
 * (sampler.h:131-134): one VOCAB_SIZE-float copy per step, same token stream. */
int qwen_decode_step(qwen_t* ctx, int token, int pos, const qwen_sampling_t* sp,
                     unsigned long long* rng_state, int* next_token);

/* n_steps chained decode steps without host round trips: step i feeds the
 * token sampled by step i-1 (step 0 feeds `token` at `pos`).  tokens_out
 * receives the n_steps sampled ids (host memory). */
int qwen_generate(qwen_t* ctx, int token, int pos, int n_steps, const qwen_sampling_t* sp,
                  unsigned long long* rng_state, int* tokens_out);

/* qwen_generate with the n_steps launches bracketed by CUDA events on the
 * handle's stream (synchronised on both sides); *device_ms receives the
 * elapsed device time.  Used by the benchmark. */
int qwen_generate_timed(qwen_t* ctx, int token, int pos, int n_steps, const qwen_sampling_t* sp,
                        unsigned long long* rng_state, int* tokens_out, float* device_ms);

/* Prompt ingestion: positions pos0 .. pos0+n-1 of `tokens` enter the KV cache
 * (no reference counterpart: the reference loops forward() per prompt
 * position, main.cu:141-145).  If logits_host is non-NULL it receives the
 * logits of the last prompt position. */
int qwen_prefill(qwen_t* ctx, const int* tokens, int n, int pos0, float* logits_host);

/* Prompt path of qwen_prefill: gemm != 0 (the default) runs prompts of 65 or
 * more tokens as whole-prompt passes on the tensor cores (every layer's
 * projections as tcgen05 GEMMs over all prompt rows, attention over the KV
 * cache), the last position's logits from an fp32 RMSNorm and LM-head GEMV
 * (with a vocabulary shard set: one decode launch for the last token instead);
 * gemm == 0 uses one decode launch per prompt token.  No reference counterpart
 * (the reference runs forward() per prompt token, main.cu:141-145). */
int qwen_set_prefill_mode(qwen_t* ctx, int gemm);

/* Precision of the tensor-core passes (qwen_prefill's long prompts and the
 * batched steps): each fp32 activation enters the bf16 GEMMs as `parts` bf16
 * terms (hi + mid + lo).  3 reproduces the fp32 product to fp32 precision; 2
 * (the default) keeps 16 mantissa bits of each activation (relative error
 * <= 2^-17) for two thirds of the tensor work, and its logits are as close to
 * the fp32 oracle as those of 3 (the bf16 K/V cache dominates the difference);
 * 1 is plain bf16 activations (about ten times further from the oracle).
 * No reference counterpart (the reference has no prompt pass). */
int qwen_set_prefill_parts(qwen_t* ctx, int parts);

/* Attention kernel of the tensor-core prompt passes: 1 (the default) the
 * tcgen05/TMEM kernel (S and O accumulated in tensor memory, K and transposed
 * V tiles by TMA, one pass over the keys with an online softmax), 0 the
 * mma.sync kernel.  Both compute the same causal attention; the environment
 * variable QWEN_B200_PREFILL_ATTN=mma selects 0 at qwen_create.  No reference
 * counterpart (the reference has no prompt pass). */
int qwen_set_prefill_attention(qwen_t* ctx, int kind);

/* Number of positions currently held in the KV cache. */
int qwen_cached_positions(const qwen_t* ctx);

/* ---- vocabulary-sharded LM head (multi-GPU, no reference counterpart) ---- */

/* Restrict this handle's LM head to vocabulary rows [row_begin, row_end).
 * qwen_shard_topk then reports the shard's top-k (logit, global id) pairs of the
 * last forward, in descending order, ties by ascending id. */
int qwen_set_vocab_shard(qwen_t* ctx, int row_begin, int row_end);
int qwen_shard_topk(qwen_t* ctx, int k, float* values_host, int* ids_host);

/* Device-resident loop of a vocabulary-sharded head (each rank one handle with
 * qwen_set_vocab_shard, all ranks the same prompt and settings).  Per token:
 * qwen_shard_decode (the trunk and the shard's rows of the LM head; the shard's
 * top-k stays on the device), qwen_shard_candidates (copies them, async on
 * the handle's stream, into the caller's device buffer), an all-gather of
 * those buffers across the ranks on the handle's stream (NCCL), then
 * qwen_shard_merge (one small kernel: merges the ranks' candidates in
 * descending order, ties by id, samples with the shared RNG state and hands the
 * token to the next qwen_shard_decode).  No host round trip until
 * qwen_shard_finish, which synchronises and returns the tokens.  Sampling
 * settings: argmax, or top-p in (0, 1) with 1 <= top_k <= 64.
 * qwen_shard_begin returns k, the candidates each rank contributes.  No
 * reference counterpart (the reference runs on one GPU). */
void* qwen_stream(qwen_t* ctx);
int qwen_shard_begin(qwen_t* ctx, int token, int pos, const qwen_sampling_t* sp, unsigned long long rng_state);
int qwen_shard_decode(qwen_t* ctx);
int qwen_shard_candidates(qwen_t* ctx, float* values_dev, int* ids_dev);
/* values_dev / ids_dev: rank r's k candidates at + r * stride (elements) */
int qwen_shard_merge(qwen_t* ctx, const float* values_dev, const int* ids_dev, int n_ranks, int stride);
int qwen_shard_finish(qwen_t* ctx, int* tokens_host, int n, unsigned long long* rng_state);

/* ---- host sampler (sampler.h) ------------------------------------------- */

/* sampler.h:120-175 on host logits, restated: argmax / top-k (Hoare quickselect)
 * / temperature softmax / top-p / inverse-CDF draw with xorshift64*.  This is
 * the reference's host API, kept for drop-in callers of sample(). */
int qwen_sample_host(const float* logits, int n, const qwen_sampling_t* sp,
                     unsigned long long* rng_state, int* token_out);

/* Merge per-shard candidate lists (values/ids, n entries, any order) into the
 * final sampled token with the device sampler's math, on the host: used after
 * the NVLink all-gather of shard top-k lists. */
int qwen_sample_candidates(const float* values, const int* ids, int n, const qwen_sampling_t* sp,
                           unsigned long long* rng_state, int* token_out);

/* ---- batched decode (no reference counterpart) ---------------------------- */
/* The reference keeps one sequence per model (its run state is batch-1,
 * qwen_model.cuh:63-80).  These serve up to 128 sequences per step on one GPU,
 * every weight read once per step for all of them: each step is one pass over
 * B rows — the projections as tensor-core GEMMs over the B rows (activations
 * in three bf16 parts, fp32-exact products), attention of each row over its own
 * cache slot in fp32, the LM head as one GEMM, top-k per row on the device and
 * the sampler's math on the host (the device sampler's, as in
 * qwen_sample_candidates; settings outside the device sampler's set, as for
 * qwen_decode_step, draw with qwen_sample_host over each whole logits row).  Same numerics as the batch-1 chain up to fp32
 * summation order. */

/* Allocates max_batch (1..128) KV cache slots, each holding SEQ_LEN positions
 * (939 MiB per slot).  Once per handle (QWEN_E_STATE after). */
int qwen_batch_init(qwen_t* ctx, int max_batch);

/* Copies the fp32 logits of the last qwen_batch_step's first `rows` rows
 * (row r is the step's sequence r; VOCAB_SIZE floats per row) to host memory. */
int qwen_batch_read_logits(qwen_t* ctx, int rows, float* logits_host);

/* Positions 0 .. n-1 of slot `slot` from `tokens` (the slot's previous
 * contents are dropped); logits_host (may be NULL) receives the last
 * position's logits. */
int qwen_batch_prefill(qwen_t* ctx, int slot, const int* tokens, int n, float* logits_host);

/* One step for slots 0 .. batch-1: row r feeds tokens[r] at position pos[r]
 * (at most the slot's current length) and returns the sampled next[r];
 * rng_states[r] is slot r's sampler state (may be NULL for greedy sampling:
 * temperature 0 or top_k 1).  Sampling as qwen_decode_step serves it
 * (1 <= top_k <= 64 unless greedy). */
int qwen_batch_step(qwen_t* ctx, int batch, const int* tokens, const int* pos, const qwen_sampling_t* sp,
                    unsigned long long* rng_states, int* next);

/* ---- tokenizer (tokenizer.h, export.py) ---------------------------------- */

typedef struct qwen_tokenizer qwen_tokenizer_t;

/* Reads a tokenizer.bin (export.py:168-244 writes it; tokenizer.h:38-70 reads
 * it): u32 max_token_length, u32 bos, u32 eos, then per token f32 merge score,
 * u32 byte length, the bytes.  vocab_size entries are read (<= 0: the model's
 * 151936); entries past the end of the file are empty, as in the reference.
 * QWEN_E_IO if the file cannot be opened, QWEN_E_FORMAT if it is truncated
 * inside an entry.  Replaces build_tokenizer's file part (tokenizer.h:38-70;
 * the prompt templates are text files the caller renders). */
int qwen_tokenizer_load(const char* path, int vocab_size, qwen_tokenizer_t** out);
void qwen_tokenizer_free(qwen_tokenizer_t* t);
int qwen_tokenizer_info(const qwen_tokenizer_t* t, int* vocab_size, int* max_token_length, int* bos, int* eos);

/* encode() (tokenizer.h:104-185): bytes -> one-byte entries ("<...>" special
 * entries first), then greedy best-score pair merges; the same token ids as the
 * reference, with hash lookups instead of linear vocabulary scans.  Writes at
 * most cap ids; *n_tokens is the full count (QWEN_E_ARG if it exceeds cap).
 * Bytes without a one-byte entry are skipped and counted in *n_unknown (may be
 * NULL); the reference leaves an unwritten slot for them. */
int qwen_tokenizer_encode(const qwen_tokenizer_t* t, const char* text, int* tokens, int cap, int* n_tokens, int* n_unknown);

/* decode() (tokenizer.h:80-82): the token's bytes as a NUL-terminated string
 * owned by the tokenizer. */
int qwen_tokenizer_decode(const qwen_tokenizer_t* t, int token, const char** piece);

/* ---- diagnostics ---------------------------------------------------------- */

/* Per-CTA ring accounting of the last decode launch: out[2c] = chunks the
 * producer issued, out[2c+1] = chunks the consumers took (they must agree).
 * Returns the number of CTAs (or a negative status). No reference counterpart. */
int qwen_debug_chunk_counts(qwen_t* ctx, int* out, int max_ctas);

/* Residual stream after every layer (resid: N_LAYERS*DIM floats) and raw
 * q|k|v projections (qkv: N_LAYERS*4096 floats) of the last launch (either may
 * be NULL).  qwen_debug_capture is kept for callers that enable capture first;
 * the values are always retained. */
int qwen_debug_capture(qwen_t* ctx, int enable);
int qwen_debug_read(qwen_t* ctx, float* resid, float* qkv);

/* Stage tracing: with tracing enabled every decode launch records %globaltimer
 * (ns) stamps per CTA at each stage boundary; qwen_trace_read copies
 * n_ctas * stride stamps of the last launch and returns their count.  The
 * stride and the meaning of each slot are documented in
 * csrc/decode_kernel.cuh (kTraceStride). */
int qwen_trace_enable(qwen_t* ctx, int enable);

/* Failure testing without a GPU fault (no reference counterpart; the
 * reference exit()s on errors, static_loader.h:22-30): every later launch
 * waits at most wait_ns (>= 1 ms; 0 restores the default 2 s) for another
 * CTA's values, and, with group >= 0, the CTAs of KV head `group` withhold
 * their layer-0 q|k|v.  The peers' waits then run out, the call returns
 * QWEN_E_TIMEOUT, the device state is reset and the KV cache invalidated;
 * qwen_debug_inject_wait(ctx, 0, -1) restores normal operation. */
int qwen_debug_inject_wait(qwen_t* ctx, unsigned long long wait_ns, int group);
int qwen_trace_read(qwen_t* ctx, unsigned long long* out, int max_entries);

/* ---- isolated kernels ---------------------------------------------------- */

/* y[n] = bf16(W[n][k] . x[k]) with fp32 accumulation; W row-major bf16, x and y
 * bf16, all device pointers (W and x 16-byte aligned); k a multiple of 256,
 * k <= 4096.  `stream` is a cudaStream_t (NULL = legacy default stream).  The
 * GEMV of matmul_cublas (qwen_model.cuh:706-757) with alpha = 1, beta = 0.
 * Asynchronous: matrices up to 64 MB take a direct-load kernel with no waits;
 * larger ones a TMA-ring kernel whose bounded waits, if one ever expires,
 * leave y invalid and set the device's error word, which
 * qwen_gemv_bf16_status reports. */
int qwen_gemv_bf16(const void* W, const void* x, void* y, int n, int k, void* stream);

/* Synchronises `stream` and reports QWEN_E_TIMEOUT if a qwen_gemv_bf16 launch
 * on the current device since the last query had a device wait expire (its y
 * is invalid), else QWEN_OK; clears the word.  Replaces the reference's
 * exit() on a failed cuBLAS call (static_loader.h:22-30). */
int qwen_gemv_bf16_status(void* stream);

/* qwen_gemv_bf16 without any device allocation.  No counterpart in the
 * reference: it is for callers that must not call cudaMalloc, such as code
 * that runs while a stream is being captured into a CUDA graph, or code inside
 * a framework whose memory pool already holds the device's memory.  (The
 * plain entry point allocates its 4-byte device error word on its first call
 * per device.)  The kernel's scratch lives in a 256-byte file-scope device
 * array that every GPU loading the library holds until exit; this call uses
 * one word of it as the ring kernel's error word, which starts at zero and is
 * read and cleared by qwen_gemv_bf16_static_status.  Same shapes, arguments
 * and result as qwen_gemv_bf16 (bit for bit): k must be a positive multiple
 * of 256 and at most 4096 (larger k is rejected with QWEN_E_ARG).  The first
 * call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  All calls share the one array, so calls whose
 * kernels overlap on the GPU race on it. */
int qwen_gemv_bf16_static(const void* W, const void* x, void* y, int n, int k, void* stream);

/* qwen_gemv_bf16_status for qwen_gemv_bf16_static's error word (allocates
 * nothing; not for use while `stream` is being captured: it synchronises). */
int qwen_gemv_bf16_static_status(void* stream);

/* C[M][N] = A[M][K] . B[N][K]^T on the tensor cores (tcgen05.mma, bf16 in, fp32
 * accumulate in TMEM; 128 x 256 or 128 x 128 tiles, TMA-fed).  A and B bf16
 * row-major (K contiguous: activations x weights in nn.Linear layout); C fp32
 * (c_fp32 != 0) or bf16, row-major.  M a multiple of 128, N of 128, K of 64;
 * all pointers device, 16-byte aligned.  The dense contraction of prefill (no
 * reference counterpart: the reference runs the decode chain per prompt token,
 * main.cu:141-145). */
int qwen_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int c_fp32, void* stream);

/* The k best entries (1 <= k <= 64) of each of `rows` rows of fp32 logits (n
 * columns, rows ld apart): values and column ids, k per row, in column order
 * (not sorted); best = larger value, ties to the smaller column; NaN ranks
 * below every number.  The device top-k of qwen_batch_step, whose candidates
 * feed the sampler's top-k (sampler.h:54-79).  All pointers device; allocates
 * scratch (4 x rows x ceil(n / 512) x k words) and synchronizes `stream`. */
int qwen_row_topk(const float* logits, int rows, int n, int ld, int k, float* values, int* ids, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_H */
