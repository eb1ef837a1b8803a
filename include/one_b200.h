/*
 * one_b200.h -- C ABI of the MedIT One B200 (sm_100a) engine, libone_b200.so.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to a
 * contiguous row-major array of the stated shape, in the model dtype unless noted
 * (ONE_DTYPE_BF16: __nv_bfloat16, ONE_DTYPE_F32: float). `stream` is a cudaStream_t
 * (NULL = legacy default stream). Every call returns ONE_OK (0) or an error code; the
 * message of the last failure on the calling thread is one_last_error(). Kernels never
 * trap: a device-side wait that runs out of time sets an error that one_engine_error()
 * reports. No call allocates device memory; callers pass workspaces sized by the
 * *_workspace_bytes functions.
 *
 * The reference (MedIT One) binds its native code as the pybind module `one_turbo`
 * (csrc/one_kernels.cpp:128-134), discovered by one/turbo_ops.py:28-93. Each legacy
 * entry point below replaces one of those five functions; the engine calls are new
 * (the reference runs the decode step op by op in PyTorch, one/modeling_one.py:325-926).
 */
#ifndef ONE_B200_H
#define ONE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ONE_B200_ABI_VERSION 2

enum { ONE_OK = 0, ONE_ERR_INVALID = 1, ONE_ERR_CUDA = 2, ONE_ERR_UNSUPPORTED = 3, ONE_ERR_DEVICE = 4 };
enum { ONE_DTYPE_BF16 = 0, ONE_DTYPE_F32 = 1 };

int one_abi_version(void);
const char* one_last_error(void);

/* ------------------------------------------------------------------ model engine */

/* The OneConfig fields the decode path reads (one/configuration_one.py:24-56).
 * num_experts = 0 selects plain nn.Linear for hx_moe / cx_moe / x_moe
 * (one/modeling_one.py:276-287). transformer_dim must equal hidden_size. */
typedef struct one_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t transformer_dim;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t head_dim;
  int32_t intermediate_size;
  int32_t num_experts;
  int32_t top_k;
  int32_t r;
  int32_t mlp_bias;
  int32_t dtype;
  float rms_norm_eps;
  float rope_theta;
  /* OneConfig.use_flash_attention (one/modeling_one.py:295-310, 408-421) with the reference's
   * turbo semantics (TurboFlashAttention(causal=True), one/turbo_ops.py:437-475): per head,
   * causal softmax attention across the call's tokens over the lin_q / lin_k / lin_v outputs
   * (head dim = num_attention_heads, scale 1/sqrt(num_attention_heads)); a one-token decode
   * call therefore sees only its own token and its attention output is lin_v(value). */
  int32_t use_flash_attention;
} one_config;

/* Per-layer weight slots (names of the reference parameters, one/modeling_one.py:231-292,
 * one/linear_moe.py:32-38). ONE_W_GATE_UP is the MLP gate_proj / up_proj pair packed
 * row-interleaved: row 2j = gate_proj row j, row 2j+1 = up_proj row j ([2*I, D]);
 * ONE_W_GATE_UP_B the same for their biases (mlp_bias only). Unused slots may be NULL. */
enum {
  ONE_W_NORM1 = 0,
  ONE_W_LIN1_W, ONE_W_LIN1_B, ONE_W_LIN2_W, ONE_W_LIN2_B, ONE_W_LIN3_W, ONE_W_LIN3_B,
  ONE_W_LINQ_W, ONE_W_LINQ_B, ONE_W_LINK_W, ONE_W_LINK_B, ONE_W_LINV_W, ONE_W_LINV_B,
  ONE_W_HX_W, ONE_W_HX_B, ONE_W_HX_GATE, ONE_W_HX_EXPERTS, ONE_W_HX_BIAS2,
  ONE_W_CX_W, ONE_W_CX_B, ONE_W_CX_GATE, ONE_W_CX_EXPERTS, ONE_W_CX_BIAS2,
  ONE_W_X_W, ONE_W_X_B, ONE_W_X_GATE, ONE_W_X_EXPERTS, ONE_W_X_BIAS2,
  ONE_W_GATE_UP, ONE_W_GATE_UP_B, ONE_W_DOWN, ONE_W_DOWN_B,
  ONE_W_NORM_W, ONE_W_NORM_B,
  ONE_W_LAYER_SLOTS
};
/* Model-level slots (one/modeling_one.py:625-658, 854). */
enum { ONE_G_EMBED = 0, ONE_G_LHS_W, ONE_G_LHS_B, ONE_G_UP_W, ONE_G_UP_B, ONE_G_NORM_W, ONE_G_NORM_B, ONE_G_LM_HEAD, ONE_G_SLOTS };

typedef struct one_engine one_engine;

/* Bytes of device workspace for an engine that runs up to max_tokens tokens per prefill
 * launch, max_batch sequences per decode step and records up to hist_cap generated tokens
 * per sequence. */
size_t one_engine_workspace_bytes(const one_config* cfg, int32_t max_tokens, int32_t max_batch, int32_t hist_cap);

/* Build an engine over caller-owned device memory: global_w[ONE_G_SLOTS],
 * layer_w[num_hidden_layers * ONE_W_LAYER_SLOTS], workspace, and two fp32 tables:
 * inv_freq [head_dim/2] (the RoPE frequencies, one/modeling_one.py:117-122) and
 * decode_div [div_len] (the running-mean divisor for each position P,
 * one/modeling_one.py:379-387: arange(1, max(P,1)+1, dtype)[-1] + 1e-10, as a float).
 * All must outlive the engine. */
int one_engine_create(const one_config* cfg, const void* const* global_w, const void* const* layer_w, void* workspace,
                      size_t workspace_bytes, int32_t max_tokens, int32_t max_batch, int32_t hist_cap,
                      const float* inv_freq, const float* decode_div, int32_t div_len, one_engine** out);
int one_engine_destroy(one_engine* e);

/* Zero the running state of `batch` sequences and set the position counter. */
int one_engine_reset(one_engine* e, int32_t batch, int32_t pos, void* stream);

/* Prompt ingestion (OneForCausalLM.forward on ids [batch, seq_len] with an empty
 * cache, one/modeling_one.py:671-926). ids: int32 [batch*seq_len]; prompt_div: fp32
 * [seq_len] divisors of the prefix mean. Leaves the running state and, for greedy
 * decode, the argmax of each sequence's last logits. logits_mode 0: none, 1: last
 * position [batch, vocab], 2: every position [batch*seq_len, vocab] into `logits`. */
int one_engine_prefill(one_engine* e, const int32_t* ids, int32_t batch, int32_t seq_len, const float* prompt_div,
                       int32_t logits_mode, void* logits, void* stream);

/* One single-token decode step for `batch` sequences (the reference's cached forward
 * with s = 1). ids: int32 [batch] input tokens, or NULL to feed each sequence the argmax
 * of its previous logits (greedy). logits: [batch, vocab] or NULL. next_ids: int32
 * [batch] argmax of this step's logits, or NULL. */
int one_engine_step(one_engine* e, int32_t batch, const int32_t* ids, void* logits, int32_t* next_ids, void* stream);

/* Capture `steps` greedy steps of `batch` sequences into a CUDA graph; replay it. */
int one_engine_capture(one_engine* e, int32_t batch, int32_t steps, void* stream);
int one_engine_replay(one_engine* e, void* stream);

/* Device pointers into the workspace (valid for the engine's lifetime). Names:
 * "state" fp32 [L][max_batch][D] running sums; "counters" int32 {pos, step};
 * "history" int32 [hist_cap][batch] greedy tokens; "hx", "cx" model dtype [max_tokens][D]
 * (the last layer's hx, cx after a forward); "router_idx" int32 [max_tokens][3][top_k]
 * (last layer's hx/x/cx experts). */
void* one_engine_buffer(one_engine* e, const char* name);
/* Nonzero when a kernel recorded a device-side error (bounded wait ran out). */
int one_engine_error(one_engine* e, int32_t* code, int32_t* where);
/* Number of kernels one_engine_step launches for `batch` sequences. */
int32_t one_engine_step_launches(one_engine* e, int32_t batch);
/* Number of kernels one_engine_prefill launches for `batch` prompts of `seq_len` tokens
 * (logits_mode as in one_engine_prefill), or -1. */
int32_t one_engine_prefill_launches(one_engine* e, int32_t batch, int32_t seq_len, int32_t logits_mode);
/* Time each launch of one decode step separately (reps back-to-back runs between two
 * CUDA events on `stream`, warm caches): us_out[i] = mean microseconds of launch i.
 * Returns the number of launches written (<= n), or -1. Advances the decode state. */
int32_t one_engine_profile_step(one_engine* e, int32_t batch, int32_t reps, float* us_out, int32_t n, void* stream);

/* ------------------------------------------------------------------ standalone ops */

/* LinearMoE.forward (one/linear_moe.py:46-99) on x [n, fin]: gate, router, the
 * reference's top-k selection (torch CPU topk with sorted=False), combine, shared
 * Linear. out [n, fout]; idx_out int32 [n, top_k] or NULL. Workspace bytes from
 * one_linear_moe_workspace_bytes. */
size_t one_linear_moe_workspace_bytes(int32_t n, int32_t fin, int32_t r, int32_t dtype);
int one_linear_moe(const void* x, int32_t n, int32_t fin, int32_t fout, const void* weight, const void* bias,
                   const void* gate_w, const void* experts, const void* bias2, int32_t num_experts, int32_t r,
                   int32_t top_k, int32_t dtype, void* out, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                   void* stream);

/* one_linear_moe without a workspace argument, for callers that cannot allocate device
 * memory: a host program that binds this library through a foreign-function interface and only
 * holds the device pointers it is handed, or a process whose device memory belongs entirely to
 * another runtime's pool. No counterpart in the reference. The scratch is a static array in the
 * library image of ONE_NOALLOC_SCRATCH_BYTES per GPU; calls needing more (n * fin too large)
 * fail with ONE_ERR_INVALID. The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress) with that device current; with CUDA's lazy module loading that lookup
 * is also when the array takes its device memory, which the GPU then holds until the process
 * exits. Make that first call before any stream capture (and, if the caller's memory is
 * budgeted, before the budget is fixed); a call made after a
 * cudaDeviceReset (a new context) looks it up again. Every call shares the
 * one array: calls whose work overlaps on the GPU (other streams, other host threads) race;
 * serialise them. No call allocates or frees device memory. */
#define ONE_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int one_linear_moe_noalloc(const void* x, int32_t n, int32_t fin, int32_t fout, const void* weight, const void* bias,
                           const void* gate_w, const void* experts, const void* bias2, int32_t num_experts, int32_t r,
                           int32_t top_k, int32_t dtype, void* out, int32_t* idx_out, void* stream);

/* Replaces one_turbo.moe_routing (csrc/one_kernels.cpp:65-74): the LinearMoE router
 * only. comb [n, fin] = mean of the selected biased inputs, idx_out [n, top_k]. */
int one_moe_routing(const void* x, int32_t n, int32_t fin, const void* gate_logits, const void* experts, const void* bias2,
                    int32_t num_experts, int32_t r, int32_t top_k, int32_t dtype, void* comb, int32_t* idx_out,
                    void* stream);

/* Replaces one_turbo.rotary_embedding (csrc/one_kernels.cpp:76-86) with the semantics of
 * OneRotaryEmbedding.forward (one/modeling_one.py:159-182): position_ids int64
 * [batch, seq], inv_freq fp32 [dim/2] -> cos, sin [batch, seq, dim] in dtype. */
int one_rotary_embedding(const int64_t* position_ids, int32_t batch, int32_t seq, const float* inv_freq, int32_t dim,
                         int32_t dtype, void* cos_out, void* sin_out, void* stream);

/* Replaces one_turbo.cumsum_and_normalize (csrc/one_kernels.cpp:88-95) with the
 * semantics of turbo_cumsum_and_normalize_cpu (one/turbo_ops.py:288-310): fp32 prefix
 * sum over dim 1 of x [b, s, d] divided by (position + 1 + 1e-8), first seq_len rows. */
int one_cumsum_and_normalize(const void* x, int32_t b, int32_t s, int32_t d, int32_t seq_len, int32_t dtype, void* out,
                             void* stream);

/* Replaces one_turbo.combined_rope_attention (csrc/one_kernels.cpp:97-125) with the
 * semantics of the model's in-line feature attention (one/modeling_one.py:515-547):
 * single_x, key, value [b, h, t, dh]; cos, sin [b or 1, t, dh]; lin_q/k/v weights
 * [hout, dh] and biases [hout] (nn.Linear layout, biases may be NULL) -> out [b, h, t, hout]. */
int one_combined_rope_attention(const void* single_x, const void* key, const void* value, const void* cos,
                                const void* sin, int32_t cos_batch, const void* wq, const void* bq, const void* wk,
                                const void* bk, const void* wv, const void* bv, int32_t b, int32_t h, int32_t t,
                                int32_t dh, int32_t hout, int32_t dtype, void* out, void* stream);

/* Replaces one_turbo.flash_attention (csrc/one_kernels.cpp:40-63) with the semantics of
 * turbo_flash_attention's PyTorch path (one/turbo_ops.py:115-143): softmax(q k^T * scale
 * [+ causal mask]) v with an fp32 softmax. q [b, h, nq, dh], k, v [b, h, nk, dh]. */
int one_flash_attention(const void* q, const void* k, const void* v, int32_t b, int32_t h, int32_t nq, int32_t nk,
                        int32_t dh, int32_t causal, float scale, int32_t dtype, void* out, void* stream);

/* The RoPE + attention operator of the isolated attention workload: apply_rotary_pos_emb_flash
 * (one/flash_attention.py:26-33) on q and k with cos, sin [cos_batch, n, dh] (cos_batch = b, or
 * 1 when shared by the batch), then exact softmax attention as one_flash_attention. q, k, v,
 * out [b, h, n, dh]. The workspace holds the rotated q and k (no reference counterpart: the
 * reference applies RoPE and attention as two Python calls). */
size_t one_rope_flash_attention_workspace_bytes(int32_t b, int32_t h, int32_t n, int32_t dh, int32_t dtype);
int one_rope_flash_attention(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                             int32_t cos_batch, int32_t b, int32_t h, int32_t n, int32_t dh, int32_t causal, float scale,
                             int32_t dtype, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Error record of the standalone ops' kernels: a bounded device-side wait that ran out
 * records its code and site here instead of trapping. Returns the code (0 = none) and the
 * site in *where (may be NULL); clears the record when clear != 0. Synchronises the device.
 * (No reference counterpart: the reference's kernels have no device-side waits.) */
int one_ops_error(int32_t* where, int32_t clear);

/* Self-test of the prompt path's prefix-mean division (a reciprocal table and one residual
 * correction instead of a division per element): every bf16 dividend (all 65536 bit
 * patterns) against each of the n divisors, compared with the fp32 division. mismatches is
 * a caller-owned DEVICE array of two counters, zeroed by the call: [0] counts fp32 results
 * that differ, [1] results that differ after rounding to bf16 (NaN equals NaN).
 * Synchronises the stream. (No reference counterpart.) */
int one_selftest_mean_division(const float* divisors, int32_t n, unsigned long long* mismatches, void* stream);

/* One token per sequence drawn from logits [batch][ld] (first `vocab` entries, model dtype),
 * warped as transformers' generation loop warps fp32 logits for do_sample=True
 * (generation/utils.py _get_logits_processor, sampling branch; transformers 5.5): scores / T,
 * then top-k (keep scores >= the k-th largest; top_k = 0: off), then top-p (keep the largest
 * tokens until their probability mass reaches top_p; top_p >= 1: off), then one draw from the
 * softmax of the kept scores. Ties at a top-k / top-p boundary are all kept. The draw for
 * sequence b uses the Philox4x32-10 counter (offset, b) under key `seed`, so equal (seed,
 * offset) give equal tokens. vocab <= 49152; temperature > 0. out [batch] int32 (device).
 * No counterpart in one_turbo: it replaces the sampling step of GenerationMixin.generate,
 * which the reference's generate() runs (one/modeling_one.py:845, README.md:73). */
int one_sample_tokens(const void* logits, int32_t batch, int32_t vocab, int32_t ld, int32_t dtype, float temperature,
                      int32_t top_k, float top_p, uint64_t seed, uint64_t offset, int32_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ONE_B200_H */
