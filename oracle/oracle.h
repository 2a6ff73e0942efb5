/*
 * CPU oracle for the ERNIE text-decoder decode step of RapidAI/RapidOCRvl.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a C++ restatement of the
 * reference's Go CPU path (internal/model/model.go + internal/tensor +
 * internal/gguf).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it, and only as the checker / CPU baseline.  The CUDA
 * product path never calls into it.
 *
 * Numerics follow the reference as compiled for amd64 with AVX-512 VNNI
 * (int8-activation dots for Q4/Q6, fp32 FMA dots for Q8 loaded from GGUF),
 * with one canonical float summation order per operation; each function in
 * oracle.cpp cites the reference file:line it restates.
 */
#ifndef OCRVL_ORACLE_H
#define OCRVL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_config {
  int vocab_size;
  int hidden_size;
  int intermediate_size;
  int num_layers;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  float rms_norm_eps;
  double rope_theta;
  int mrope_section[3];
} orc_config;

/* Tensor types as stored in the repo's GGUF files (internal/gguf/gguf.go:19-22). */
enum { ORC_F32 = 0, ORC_Q8 = 1000, ORC_Q4 = 1001, ORC_Q6 = 1002 };

/* ---- model / sequence --------------------------------------------------- */
void *orc_load(const char *gguf_path, const orc_config *cfg, char *err, int errlen);
void orc_free(void *model);
/* OpenMP threads of the oracle's parallel loops (n > 0 sets them); returns
 * the count in effect.  The CPU baseline sets every host core. */
int orc_set_threads(int n);
int orc_quant_type(void *model);
void *orc_seq_new(void *model, int max_tokens);
void orc_seq_free(void *seq);
int orc_seq_len(void *seq);
/* Copies layer `layer`'s K and V caches ([len][kv_heads*head_dim] f32). */
int orc_seq_kv(void *seq, int layer, float *k, float *v);
/* Replaces the cache with n positions given for every layer
 * ([num_layers][n][kv_heads*head_dim] f32 each) and sets the length to n. */
int orc_seq_import_kv(void *seq, int n, const float *k, const float *v);

/* One decode step (Runtime.forwardEmbeddingForSampling, model.go:3475-3643).
 * emb: hidden_size f32.  pos: (T,H,W).  If need_logits, writes the argmax id to
 * *token (ties -> lowest id) and, if logits != NULL, the full logits.
 * final_norm (nullable) receives the lm_head input vector. */
int orc_forward(void *model, void *seq, const float *emb, int pT, int pH, int pW,
                int need_logits, int *token, float *logits, float *final_norm);

/* orc_forward with need_logits, also writing the intermediates of every
 * layer to dump: [h_in H | norm1 H | q QH*D | k KVH*D | v KVH*D (before RoPE)
 * | head QH*D | h + o H | norm2 H | g I] per layer (debugging aid). */
int orc_forward_dump(void *model, void *seq, const float *emb, int pT, int pH, int pW, int *token,
                     float *logits, float *dump);

/* Greedy generation (Runtime.GenerateWithOptions, model.go:1492-1572) with
 * temperature 0.  out receives prompt + generated ids; returns count or <0. */
int orc_generate(void *model, const int *ids, int n_ids, int max_new,
                 const int *eos, int n_eos, int *out, int out_cap);

/* Decode-only timing helper for the CPU baseline: runs `steps` greedy decode
 * steps on `seq` starting from token `tok` at position `pos`; returns the
 * last token. */
int orc_decode_steps(void *model, void *seq, int tok, int pos, int steps);

/* Embedding row gather (tokenEmbeddingInto, model.go:3251-3258). */
int orc_embed(void *model, int id, float *out);

/* ---- op level ----------------------------------------------------------- */
/* Row quantizers used by the GGUF converter (quant.go:96-137, 201-384). */
float orc_quantize_row(int type, const float *w, int cols, uint8_t *packed);
/* Unpack one packed row to int8 (quant.go:2325-2368, 2605-2656). */
void orc_unpack_row(int type, const uint8_t *packed, int cols, int8_t *out);
/* quantizeXForVNNI (quant.go:2087-2115, dot_vnni_amd64.s:434-500). */
float orc_quantize_x(const float *x, int n, uint8_t *xq);
/* dotQ8VNNICore (dot_vnni_amd64.s): sum of w[i] * xq[i] in int32. */
int32_t orc_dot_u8s8(const int8_t *w, const uint8_t *xq, int n);
/* finalizeDotQ8VNNI lane (dot_vnni_amd64.s:1043-1090). */
float orc_vnni_finalize(int32_t dot, int32_t rowsum, float scale_x, float scale_w);
/* dotQ8 fp32 FMA order (quant.go:2062-2198), unscaled. */
float orc_dot_q8_f32(const int8_t *w, const float *x, int n);
/* matVecMaybeQuant semantics per type: Q4/Q6 via int8 activations, Q8 via
 * fp32 FMA dots.  data = packed rows as stored in GGUF. */
void orc_matvec(int type, int rows, int cols, const float *scales, const void *data,
                const float *x, float *out);
/* Fused matvec + residual + RMSNorm (fused_matvec2.go).  in_place=1 updates
 * residual (MatVec*AddRMSNorm), 0 leaves it (…OutOnly). */
void orc_matvec_add_rmsnorm(int type, int rows, int cols, const float *scales,
                            const void *data, const float *x, float *residual,
                            const float *norm_w, float eps, int in_place, float *norm_out);
/* SwiGLU gate/up (quant.go:757-1000 + ops.go:1125-1138). */
void orc_swiglu(int type, int rows, int cols, const float *gs, const void *gd,
                const float *us, const void *ud, const float *x, float *out);
void orc_rmsnorm(const float *x, const float *w, int n, float eps, float *out);
float orc_fast_rsqrt(float x);
float orc_fast_exp(float x);
void orc_rope(float *x, int heads, int dim, const float *cos_t, const float *sin_t);
void orc_rope_table(const orc_config *cfg, int pT, int pH, int pW, float *cos_t, float *sin_t);
void orc_softmax(float *x, int n);
/* Decode attention over a contiguous cache ([n][kv_heads*dim]) for all heads. */
void orc_attention(const float *q, const float *kc, const float *vc, int n, int heads,
                   int kv_heads, int dim, float *head_out);
int orc_argmax_matvec(int type, int rows, int cols, const float *scales, const void *data,
                      const float *x, float *best_score);
/* ---- sampling (model.go:1821-2828, topk.go, cumsum.go) ------------------ */
/* fastRNG.Float64 (model.go:1833-1840): advances *state, returns [0, 1). */
double orc_rng_float64(uint64_t *state);
/* topKSelectWithWork (topk.go:326-347): the k highest scores (ties -> lower
 * id), descending. */
void orc_topk_select(const float *logits, int n, int k, int *ids, float *scores);
/* sampleCandidateScoresScratch (model.go:1929-1976) on k candidates. */
int orc_sample_candidates(const int *ids, const float *scores, int k, double temperature, uint64_t *state);
/* pickCumulativeFloat32 (model.go:2326-2340): first index with pick <=
 * cdf[i] by binary search, or -1. */
int orc_pick_cumulative(const float *cdf, int n, float pick);
/* sampleFullLogitsScratch with a weight scratch (model.go:2215-2307);
 * -2 unless n is a multiple of 16 (>= 16). */
int orc_sample_full(const float *logits, int n, float temperature, uint64_t *state);
/* The generation loop's sampler: argmax for temperature <= 0 or top_k == 1,
 * top-k candidates for 2 <= top_k < n, else the full logits. */
int orc_sample_token(const float *logits, int n, double temperature, int top_k, uint64_t *state);
/* GenerateWithOptions with sampling; the RNG starts at uint64(seed). */
int orc_generate_sampled(void *model, const int *ids, int n_ids, int max_new, const int *eos, int n_eos,
                         double temperature, int top_k, int64_t seed, int *out, int out_cap);

#ifdef __cplusplus
}
#endif
#endif
