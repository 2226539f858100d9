/*
 * lastro_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's CPU decode path (brenoperucchi/lastro-rust,
 * rust/moe-rt/src/{cpu.rs,block.rs,model.rs,pool.rs}).  It is the checker for the
 * CUDA library and the timed CPU baseline; it is never linked into the product
 * (liblastro_b200.so) and the product never calls it.
 *
 * Numerics follow the reference function by function (each definition in
 * lastro_oracle.c cites the file:line it restates): weights are bf16 widened by a
 * 16-bit shift, activations/accumulators are f32, the dot product keeps the
 * reference's 4x8-lane FMA accumulator order, every other expression is evaluated
 * without contraction (compile with -ffp-contract=off), and exp/pow/sin/cos come
 * from the platform libm as Rust's f32 methods do on Linux.
 *
 * The synthetic generator (lo_synth_*) is shared with the CUDA library's device
 * fill kernel: integer hashing plus one exact f32 multiply, so host and device
 * produce bit-identical weights for the same (seed, index).
 */
#ifndef LASTRO_ORACLE_H
#define LASTRO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- synthetic data (shared formula with the device fill kernel) ---------- */
uint64_t lo_mix64(uint64_t z);
uint64_t lo_tensor_seed(uint64_t base, int32_t layer, int32_t kind);
/* value of element idx: (sum of four 16-bit hash chunks - 131070) * scale,
 * an Irwin-Hall(4) approximation of N(0, scale*37837.23). */
float lo_synth_value(uint64_t seed, uint64_t idx, float scale);
float lo_synth_scale(float stddev);
void lo_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float stddev, float mean, int threads);
void lo_synth_f32(float *out, size_t n, uint64_t seed, float stddev, float mean, int threads);
void lo_synth_tokens(int32_t *out, size_t n, uint64_t seed, int32_t vocab);
void lo_ref_values(float *out, size_t n, uint64_t seed);
uint16_t lo_f32_to_bf16(float f);
float lo_bf16_to_f32(uint16_t b);

/* ---- Q8_0 (no reference implementation) --------------- */
/* a row of cols weights (cols a multiple of 32) is cols/32 blocks of 34 bytes: the fp16 scale, then 32 int8 values;
 * weight = scale * value (exact in f32).  The oracle's path is the dequantised one. */
enum { LO_W_BF16 = 0, LO_W_Q8_0 = 1 };
uint16_t lo_f32_to_f16(float f);
float lo_f16_to_f32(uint16_t h);
int8_t lo_synth_q8_value(uint64_t seed, uint64_t idx);
uint16_t lo_synth_q8_scale(uint64_t seed, uint64_t block);
void lo_synth_q8_0(uint8_t *out, size_t rows, size_t cols, uint64_t seed, int threads);
size_t lo_row_bytes(int32_t dtype, size_t cols);
float lo_dot_q8(const uint8_t *row, const float *x, size_t n);
float lo_dot_q8_portable(const uint8_t *row, const float *x, size_t n);

/* ---- thread pool (pool.rs: fixed workers, tasks claimed by an atomic counter) */
typedef struct lo_pool lo_pool;
lo_pool *lo_pool_create(int threads);
void lo_pool_destroy(lo_pool *p);
int lo_pool_threads(const lo_pool *p);

/* ---- kernels of the CPU path --------------------------------------------- */
float lo_dot(const uint16_t *w, const float *x, size_t n);          /* cpu.rs:54-62 */
float lo_dot_portable(const uint16_t *w, const float *x, size_t n); /* same order, no SIMD */
void lo_gemv(lo_pool *p, const uint16_t *w, int32_t rows, int32_t cols, const float *x, float *y);
void lo_gemv_w(lo_pool *p, int32_t dtype, const void *w, int32_t rows, int32_t cols, const float *x, float *y);
void lo_swiglu(const float *h, int32_t inter, float *a);
void lo_routing(const float *logits, int32_t e, int32_t k, int32_t *ids, float *weights);
void lo_experts(lo_pool *p, const float *x, int32_t k, const uint16_t *const *gate_up,
                const uint16_t *const *down, const float *weights, int32_t hidden, int32_t inter,
                float *y);
void lo_experts_w(lo_pool *p, int32_t dtype, const float *x, int32_t k, const void *const *gate_up,
                  const void *const *down, const float *weights, int32_t hidden, int32_t inter, float *y);
/* HostLayer::forward_cpu: router [E,H], gate_up [E,2I,H], down [E,H,I] */
void lo_block_forward(lo_pool *p, const uint16_t *router, const uint16_t *gate_up,
                      const uint16_t *down, int32_t experts, int32_t hidden, int32_t inter,
                      int32_t k, const float *x, float *y, int32_t *ids, float *weights,
                      float *logits_or_null);
void lo_block_forward_w(lo_pool *p, int32_t dtype, const void *router, const void *gate_up, const void *down,
                        int32_t experts, int32_t hidden, int32_t inter, int32_t k, const float *x, float *y,
                        int32_t *ids, float *weights, float *logits_or_null);
void lo_rmsnorm(const float *x, const float *w, int32_t n, float eps, float *out);
void lo_rope_cos_sin(float theta, int32_t head_dim, int32_t pos, float *cs);
void lo_rope(float *x, int32_t n, int32_t d, const float *cs);
int32_t lo_argmax_last(const float *v, int32_t n);
int lo_total_cmp(float a, float b);

/* ---- whole model (model.rs) ------------------------------------------------ */
typedef struct {
    int32_t hidden, inter, layers, heads, kv_heads, head_dim, vocab, experts, k;
    float rope_theta, eps, embedding_multiplier, residual_multiplier, attention_multiplier,
        logits_scaling;
    int32_t weight_dtype; /* LO_W_BF16 or LO_W_Q8_0: the linear weights (embeddings and norms are bf16 / f32) */
} lo_config;

typedef struct {
    const float *ln_attn, *ln_moe; /* [H] */
    const void *q, *k, *v, *o;     /* [qd,H] [kvd,H] [kvd,H] [H,qd], of the config's weight type */
    const void *router;            /* [E,H] */
    const void *gate_up;           /* [E,2I,H] */
    const void *down;              /* [E,H,I] */
} lo_layer_weights;

typedef struct lo_model lo_model;
/* weights are borrowed (caller keeps them alive): embed [V,H], norm [H], layers[L] */
lo_model *lo_model_create(const lo_config *cfg, const uint16_t *embed, const float *norm,
                          const lo_layer_weights *layers);
/* allocates and fills every tensor from the synthetic generator (owned by the model) */
lo_model *lo_model_create_synthetic(const lo_config *cfg, uint64_t seed, float stddev,
                                    float norm_std, int threads);
/* router logit bias [layers, experts] added before every layer's routing (NULL: none); copied */
void lo_model_set_router_bias(lo_model *m, const float *bias);
void lo_model_destroy(lo_model *m);
const lo_config *lo_model_config(const lo_model *m);
const void *lo_model_tensor(const lo_model *m, int32_t layer, int32_t kind);

typedef struct lo_session lo_session;
lo_session *lo_session_create(const lo_model *m, lo_pool *p, int32_t max_len);
void lo_session_destroy(lo_session *s);
/* K/V rows rounded to bf16 (RNE) when stored: the arithmetic of a paged bf16 KV cache (off by default) */
void lo_session_set_kv_bf16(lo_session *s, int32_t on);
/* router logits [layers, experts] of the session's last step (bias included) */
const float *lo_session_router_logits(const lo_session *s);
void lo_session_reset(lo_session *s);
int32_t lo_session_pos(const lo_session *s);
/* CpuSession::step: logits [V]; ids/weights [L*k] may be NULL. Returns 0, or -1 when full. */
int lo_session_step(lo_session *s, int32_t token, float *logits, int32_t *ids, float *weights);
/* CpuSession::step in phases (the batched expert-parallel restatement runs the MoE block itself): begin (embedding;
 * -1 when full or the token is out of range), then for every layer in order the attention half (xn_out [H] = the
 * MoE block's input) and the MoE half (x += residual_multiplier * y), then end (logits [V]; the position advances).
 * lo_session_step is these phases with the block in between. */
int lo_session_step_begin(lo_session *s, int32_t token);
void lo_session_layer_attention(lo_session *s, int32_t layer, float *xn_out);
/* the residual stream of the step in progress [H] (between phases) */
void lo_session_residual(const lo_session *s, float *out);
void lo_session_layer_moe(lo_session *s, int32_t layer, const float *y);
void lo_session_step_end(lo_session *s, float *logits);
/* append synthetic K/V rows (tests/bench only: a context of `n` positions without running the model) */
int lo_session_fill_kv(lo_session *s, int32_t n, uint64_t seed, float stddev);
/* the K/V cache of layer l as [pos, kvd] f32 */
const float *lo_session_k(const lo_session *s, int32_t layer);
const float *lo_session_v(const lo_session *s, int32_t layer);

/* tensor kinds for lo_tensor_seed / lo_model_tensor */
enum {
    LO_T_EMBED = 0, LO_T_NORM = 1,
    LO_T_LN_ATTN = 2, LO_T_LN_MOE = 3, LO_T_Q = 4, LO_T_K = 5, LO_T_V = 6, LO_T_O = 7,
    LO_T_ROUTER = 8, LO_T_GATE_UP = 9, LO_T_DOWN = 10
};

#ifdef __cplusplus
}
#endif
#endif
