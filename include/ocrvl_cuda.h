/*
 * ocrvl_cuda.h -- C ABI of the B200 (sm_100a) decode path for the ERNIE text
 * decoder of RapidAI/RapidOCRvl (Go module paddleocrvl-go).
 *
 * The ABI is what a cgo shim behind the reference's backend interface binds:
 * plain pointers and sizes, no CUDA or torch types.  Each entry point names
 * the reference interface it replaces (paths relative to the reference root).
 *
 * Conventions
 *   - Every function returns OCRVL_OK (0) or a negative OCRVL_E_* code;
 *     ocrvl_last_error() then describes the failure (thread-local string).
 *   - Host pointers are only read or written during the call; nothing is
 *     retained (cgo pointer rules).
 *   - A model handle may be used from several threads; calls on it are
 *     serialised internally.  There is no CPU fallback: every compute entry
 *     point fails when the GPU path cannot run.
 *   - Tensor types: 0 = F32, 1000 = Q8_ROW, 1001 = Q4_ROW, 1002 = Q6_ROW
 *     (internal/gguf/gguf.go:19-22).  Quantized tensors are passed exactly
 *     as stored in the repo's GGUF files: rows f32 scales, then rows packed
 *     rows (internal/gguf/gguf.go:435-569).
 */
#ifndef OCRVL_CUDA_H
#define OCRVL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OCRVL_OK 0
#define OCRVL_E_INVALID (-1)  /* bad argument, shape or state */
#define OCRVL_E_CUDA (-2)     /* CUDA runtime error or no device */
#define OCRVL_E_NOMEM (-3)    /* device memory or KV pages exhausted */
#define OCRVL_E_TIMEOUT (-4)  /* a bounded device-side wait gave up */

#define OCRVL_F32 0
#define OCRVL_Q8_ROW 1000
#define OCRVL_Q4_ROW 1001
#define OCRVL_Q6_ROW 1002

typedef struct ocrvl_model ocrvl_model;
typedef struct ocrvl_seq ocrvl_seq;

/* Decoder shape, mirroring internal/config/config.go:31-49 after Load's
 * defaults.  kv_pool_bytes: device memory for paged f32 KV (0 = 4 GiB).
 * max_position: largest RoPE position + 1 (0 = 32768). */
typedef struct ocrvl_model_desc {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_layers;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float rms_norm_eps;
  double rope_theta;
  int32_t mrope_section[3];
  int32_t max_position;
  int64_t kv_pool_bytes;
} ocrvl_model_desc;

/* Last error message of the calling thread ("" if none). */
const char *ocrvl_last_error(void);

/* Number of visible CUDA devices (internal/backend/backend.go:85-111 gains a
 * "cuda" choice; this is its probe).  Returns >= 0 or OCRVL_E_CUDA. */
int ocrvl_device_count(void);

/* Creates an empty model on `device`.  Replaces the Runtime construction in
 * model.LoadWithOptions (internal/model/model.go:546-605). */
int ocrvl_init(int device, const ocrvl_model_desc *desc, ocrvl_model **out);

/* Uploads one tensor.  Replaces preloadTextWeights' per-tensor load
 * (internal/model/model.go:2861-2945): `scales` is NULL for F32, `data` the
 * packed rows (or f32 values).  Names other than the decoder's are ignored. */
int ocrvl_load_tensor(ocrvl_model *m, const char *name, int type, int64_t rows, int64_t cols,
                      const float *scales, const void *data);

/* Loads every decoder tensor of a GGUF file (gguf.Open + Q*Row / Float32,
 * internal/gguf/gguf.go:111-569) through ocrvl_load_tensor. */
int ocrvl_load_gguf(ocrvl_model *m, const char *path);

/* Checks that all decoder tensors are present and prepares the device state
 * (row sums, RoPE tables, work buffers).  Required before any step. */
int ocrvl_finalize(ocrvl_model *m);

/* Quantization type of the loaded linear weights (OCRVL_Q*_ROW) or < 0. */
int ocrvl_quant_type(const ocrvl_model *m);

/* Step trace (no reference counterpart; the reference only has load-phase
 * timings, internal/model/model.go:503-509).  With OCRVL_TRACE set at
 * ocrvl_finalize, the step kernel records per phase [start, prologue end,
 * end (max over blocks), barrier exit] as %globaltimer ns; this copies up to
 * cap values of the last step and clears them.  Returns the count (0 when
 * tracing is off). */
int ocrvl_trace_read(ocrvl_model *m, uint64_t *out, int cap);

/* Polls a block of the step kernel makes at a grid barrier before it gives up
 * (0 restores the default, about 4 million).  A step whose barrier wait runs
 * out returns OCRVL_E_TIMEOUT, leaves its sequences as they were (no position
 * appended) and resets the device barrier state, so the next step runs
 * normally.  No reference counterpart: the reference detects failures by op
 * error returns (internal/model/model.go:7235-7285); this bounds the device
 * waits that replace them, and a small limit lets a test exercise the
 * timeout path without faulting the GPU. */
int ocrvl_set_wait_limit(ocrvl_model *m, int64_t barrier_polls);

/* Copies up to `count` floats of one of the step's work buffers, as the
 * last step left them, to host memory (no reference counterpart: a
 * debugging aid for comparing a step's intermediates with a CPU run).
 * which: 0 residual h [n][hidden], 1 residual + projection [n][hidden], 2 q|k|v
 * before RoPE [n][(heads + 2 kv_heads) head_dim], 3 attention output
 * [n][heads head_dim], 4 SwiGLU output [n][intermediate], 5 long-cache
 * attention scores (per sequence [kv head][head][positions], sequences in
 * order); each for the last layer the step ran.  Returns the number of floats
 * copied. */
int ocrvl_debug_read(ocrvl_model *m, int which, float *out, int64_t count);

void ocrvl_free(ocrvl_model *m);

/* A decode sequence owning paged KV for up to max_tokens positions.
 * Replaces getKVCaches/putKVCaches (internal/model/model.go:3286-3344). */
int ocrvl_seq_create(ocrvl_model *m, int max_tokens, ocrvl_seq **out);
int ocrvl_seq_reset(ocrvl_seq *s);
void ocrvl_seq_free(ocrvl_seq *s);
int ocrvl_seq_len(const ocrvl_seq *s);

/* Copies layer `layer`'s cached K and V ([len][kv_heads*head_dim] f32 each,
 * the contiguous kvCache layout of model.go:373-379) to host memory,
 * gathering through the sequence's block table. */
int ocrvl_seq_read_kv(ocrvl_seq *s, int layer, float *k, float *v);

/* Replaces the sequence's cache with n positions of K and V given for every
 * layer ([num_layers][n][kv_heads*head_dim] f32 each, the layout
 * ocrvl_seq_read_kv returns) and sets its length to n; the next step
 * continues at position n.  No reference counterpart: it restores a cache
 * saved with ocrvl_seq_read_kv (or built elsewhere) without replaying the
 * prompt, e.g. to set up long contexts for profiling.  Invalid arguments
 * leave the sequence unchanged; a later failure (page pool exhausted, copy
 * error) leaves it empty. */
int ocrvl_seq_import_kv(ocrvl_seq *s, int n, const float *k, const float *v);

/* Sets the sequence's cache to n positions of seeded pseudo-random K and V
 * generated on the device (K uniform in [-0.5, 0.5), V in [-1, 1), a hash of
 * seed, position, layer, kv head and dim) and its length to n.  No reference
 * counterpart: it stands in for a prompt's prefill when only the decode steps
 * after it are measured (long-prompt benchmarks), without a host copy of the
 * cache.  Errors leave the sequence empty. */
int ocrvl_seq_fill_synthetic(ocrvl_seq *s, int n, uint64_t seed);

/* One decode step for n sequences (1 <= n <= 64) of the same model: the
 * batched form of Runtime.forwardEmbeddingForSampling
 * (internal/model/model.go:3475-3643).  Every sequence is validated before
 * any state changes; the step then runs as one kernel launch per group of up
 * to 8 sequences.
 *   ids       n token ids (embedding rows), or NULL when embeds is given
 *   embeds    n*hidden_size f32 input embeddings, or NULL
 *   pos_thw   n*3 M-RoPE positions, or NULL for (len, len, len)
 *   need_logits  0: prompt token (K/V only in the last layer), 1: full step
 *   out_ids   n greedy ids (lm_head argmax, ties -> lowest id), may be NULL
 *   out_logits  n*vocab_size f32 logits, may be NULL
 * When the step runs as several launches (Q8, or more than 8 sequences
 * without the batched kernel) and a later launch fails (timeout or CUDA
 * error), the sequences of the earlier launches have already taken the step:
 * ocrvl_seq_len tells the caller which ones advanced. */
int ocrvl_step(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
               const int32_t *pos_thw, int need_logits, int32_t *out_ids, float *out_logits);

/* Greedy generation (Runtime.GenerateWithOptions with temperature 0,
 * internal/model/model.go:1492-1572): prompt tokens one at a time, then up to
 * max_new tokens, stopping after an EOS id (eos NULL -> {2}).  out receives
 * prompt + generated ids; *n_out their count. */
int ocrvl_generate_greedy(ocrvl_model *m, const int32_t *ids, int n_ids, int max_new, const int32_t *eos,
                          int n_eos, int32_t *out, int out_cap, int *n_out);

/* One decode step (as ocrvl_step with need_logits = 1) whose next ids are
 * drawn by the reference's generation-loop sampler on its CPU backend
 * (Runtime.GenerateWithOptions' sampling, internal/model/model.go:1536-1544,
 * 3611-3642, 7202-7233), on the device from the step's logits:
 *   temperature <= 0 or top_k == 1  argmax (ocrvl_step's greedy id, no draw)
 *   2 <= top_k < vocab_size         the top_k logits, ties to the lower id,
 *       in descending order (MatVecTopK*WithWork, internal/tensor/topk.go:
 *       326-347), drawn by sampleCandidateScoresScratch (model.go:1929-1976);
 *       top_k <= 4096
 *   top_k == 0 or >= vocab_size     the full logits (sampleFullLogitsScratch,
 *       model.go:2215-2307); vocab_size must be a multiple of 16
 * rng_state: n fastRNG states (model.go:1829-1852), one per sequence, each
 * advanced by one draw per sampled token; NULL only for argmax.  A negative
 * temperature counts as 0 (the reference validates it before generation). */
int ocrvl_step_sample(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *ids, const float *embeds,
                      const int32_t *pos_thw, double temperature, int top_k, uint64_t *rng_state, int32_t *out_ids);

/* Runtime.GenerateWithOptions (internal/model/model.go:1492-1572): greedy as
 * ocrvl_generate_greedy when temperature <= 0 or top_k == 1, else sampled
 * through ocrvl_step_sample with one RNG started at uint64(seed)
 * (samplingRNGInto, model.go:1846-1852). */
int ocrvl_generate(ocrvl_model *m, const int32_t *ids, int n_ids, int max_new, const int32_t *eos, int n_eos,
                   double temperature, int top_k, int64_t seed, int32_t *out, int out_cap, int *n_out);

/* Greedy decode of `steps` tokens for n sequences with the token feedback
 * kept on the device (the decode loop of GenerateWithOptions,
 * internal/model/model.go:1538-1568, without the per-token EOS check): the
 * step kernel writes each argmax id and advances its own parameters, so no
 * host round trip happens between tokens.  first_ids: the n ids to feed
 * first; out_ids: steps*n generated ids (step-major), 1 <= n <= 64 (groups
 * of up to 8 sequences run one after another).  KV pages for all steps are
 * reserved before the first launch. */
int ocrvl_decode_greedy_device(ocrvl_model *m, ocrvl_seq *const *seqs, int n, const int32_t *first_ids, int steps,
                               int32_t *out_ids);

/* The model's CUDA stream (a cudaStream_t) for callers that time or order
 * work against the engine's launches; no reference counterpart. */
void *ocrvl_model_stream(ocrvl_model *m);

/* Host<->device bytes one ocrvl_step call of n sequences moves besides
 * embeddings and logits (step parameters in, ids and status out; 1 <= n <= 64). */
int ocrvl_step_io_bytes(const ocrvl_model *m, int n, int64_t *h2d, int64_t *d2h);

/* ---- op level: device pointers, optional cudaStream_t as void* --------
 * Kernel-level entry points for parity tests and for callers that hold
 * their own device buffers; each names the internal/tensor function whose
 * result it reproduces.  Quantized matrices: w = packed rows (rows x
 * packed_row_bytes), scale = rows f32, rowsum = rows int32 from
 * ocrvl_op_rowsum.  m = number of input vectors (1..8). */

/* Per-row sum of the unpacked int8 weights (UnpackQ4Matrix / UnpackQ6Matrix
 * RowSum, internal/tensor/quant.go:2325-2368, 2605-2656). */
int ocrvl_op_rowsum(int type, int rows, int cols, const void *w, int32_t *rowsum, void *stream);

/* out[m][rows] = W x[m]  (tensor.MatVecQ8/Q4/Q6, quant.go:443-561).
 * norm_w != NULL first applies RMSNorm(x, norm_w, eps) (ops.go:1015-1037). */
int ocrvl_op_matvec(int type, int rows, int cols, const void *w, const float *scale,
                    const int32_t *rowsum, int m, const float *x, const float *norm_w, float eps,
                    float *out, void *stream);

/* v = residual + W x; residual = v when in_place; norm_out = RMSNorm of v with
 * the fused sum-of-squares order (tensor.MatVec*AddRMSNorm[OutOnly],
 * internal/tensor/fused_matvec2.go). */
int ocrvl_op_matvec_add_rmsnorm(int type, int rows, int cols, const void *w, const float *scale,
                                const int32_t *rowsum, int m, const float *x, float *residual,
                                int in_place, const float *norm_w, float eps, float *v_out,
                                float *norm_out, void *stream);

/* out = silu(Wg x) * (Wu x)  (tensor.SwiGLUGateUp*Scratch, quant.go:757-1000). */
int ocrvl_op_swiglu(int type, int rows, int cols, const void *wg, const float *sg, const int32_t *rsg,
                    const void *wu, const float *su, const int32_t *rsu, int m, const float *x,
                    float *out, void *stream);

/* ids[m] = argmax_r (W x[m])_r, first maximum (tensor.MatVecArgmaxQ*,
 * internal/tensor/argmax_quant.go). */
int ocrvl_op_argmax(int type, int rows, int cols, const void *w, const float *scale,
                    const int32_t *rowsum, int m, const float *x, int32_t *ids, void *stream);

/* The same argmax as ocrvl_op_argmax for callers that must not allocate
 * device memory (no counterpart in the reference).  ocrvl_op_argmax
 * cudaMalloc's a small key buffer on first use; a server that has reserved the
 * GPU's memory for its own pools, or a loop that cannot afford the device
 * synchronisation cudaMalloc may cause, uses this variant, which keeps the keys
 * in a fixed static device array and allocates nothing.  Limit: m <= 8
 * vectors (64 bytes of keys); larger m returns OCRVL_E_INVALID.  The first
 * call on a device looks up the array's device address; make it before any
 * stream capture.  Every call clears and reuses the same array, so calls that
 * overlap on the GPU (other streams or threads on the same device) race and
 * must be ordered by the caller. */
int ocrvl_op_argmax_noalloc(int type, int rows, int cols, const void *w, const float *scale,
                            const int32_t *rowsum, int m, const float *x, int32_t *ids, void *stream);

/* The sampler of ocrvl_step_sample on m rows of logits ([m][vocab] device
 * floats): out_ids[m], rng_state[m] (device uint64, advanced), optional
 * cand_ids / cand_scores ([m][top_k], top-k path only: the candidates in the
 * order sampleCandidateScoresScratch sees them), work ([m][vocab] floats,
 * full-vocabulary path only; logits and work 16-byte aligned there).  No
 * allocation. */
int ocrvl_op_sample(int m, int vocab, const float *logits, double temperature, int top_k, uint64_t *rng_state,
                    int32_t *out_ids, int32_t *cand_ids, float *cand_scores, float *work, void *stream);

/* out = RMSNorm(x, w, eps) for m vectors of n (tensor.RMSNorm). */
int ocrvl_op_rmsnorm(int n, int m, const float *x, const float *w, float eps, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* OCRVL_CUDA_H */
