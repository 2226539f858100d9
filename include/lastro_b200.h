/*
 * lastro_b200.h -- C ABI of the B200-native Granite-MoE decode library (liblastro_b200.so).
 *
 * Drop-in boundary for the GPU operator API of brenoperucchi/lastro-rust
 * (rust/moe-rt).  Every entry point below names the reference item it replaces
 * (file:line inside that project).  Plain pointers and sizes only; host buffers
 * are caller-owned and only read/written during the call.
 *
 * Status codes follow the reference's error policy (gpu_model.rs:249-267,
 * gpu.rs:345-355):
 *   - argument errors are refused before any launch and leave the object usable;
 *   - a CUDA runtime error synchronizes the stream, then poisons the object:
 *     every later call on it returns LASTRO_E_POISONED.
 * One caller thread per object (the reference's &mut self).
 */
#ifndef LASTRO_B200_H
#define LASTRO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LASTRO_OK 0
#define LASTRO_E_ARG 1         /* bad argument or shape: refused before any launch */
#define LASTRO_E_CUDA 2        /* CUDA runtime error: stream synchronized, object poisoned */
#define LASTRO_E_POISONED 3    /* object unusable after an earlier runtime error */
#define LASTRO_E_FULL 4        /* KV cache full (gpu_model.rs:252-254) */
#define LASTRO_E_NOMEM 5       /* device allocation failed */
#define LASTRO_E_UNSUPPORTED 6 /* shape/dtype outside what the kernels implement */
#define LASTRO_E_STATE 7       /* e.g. a weight tensor not loaded yet */
#define LASTRO_E_IO 8          /* a file could not be opened or read (WeightError::Io, weights.rs:26-29) */

#define LASTRO_DTYPE_BF16 1
#define LASTRO_DTYPE_F32 2
/* Q8_0 (no reference implementation): along each row, blocks of 32 weights stored as 34 bytes --
 * the block's fp16 scale, then 32 int8 values; weight = scale * value.  A model created with weight_dtype Q8_0 takes
 * every linear weight (q/k/v/o projections, router, experts) in this layout; embeddings stay bf16, norms bf16/f32. */
#define LASTRO_DTYPE_Q8_0 3

typedef struct lastro_ctx lastro_ctx;
typedef struct lastro_layer lastro_layer;
typedef struct lastro_model lastro_model;

/* model.rs:14-31 Config (+ the dtypes the device keeps) */
typedef struct {
    int32_t hidden, inter, layers, heads, kv_heads, head_dim, vocab, experts, k;
    float rope_theta, eps, embedding_multiplier, residual_multiplier, attention_multiplier, logits_scaling;
    int32_t weight_dtype; /* LASTRO_DTYPE_BF16 or LASTRO_DTYPE_Q8_0 (linear weights) */
    int32_t kv_dtype;     /* LASTRO_DTYPE_BF16 (paged bf16 KV) or LASTRO_DTYPE_F32 */
} lastro_model_desc;

/* ---- context: one device, one stream (the reference's Arc<Stream>, gpu.rs:333) ---------------------------------- */
/* stream_or_null: a cudaStream_t to enqueue on, or NULL for a stream owned by the context */
int lastro_ctx_create(int32_t device, void *stream_or_null, lastro_ctx **out);
/* the context lives on until its last layer and model are destroyed: objects may be destroyed in any order */
void lastro_ctx_destroy(lastro_ctx *ctx);
int lastro_ctx_synchronize(lastro_ctx *ctx);
/* text of the last error on this context ("" if none); valid until the next call on ctx */
const char *lastro_last_error(const lastro_ctx *ctx);
const char *lastro_version(void);

/* ---- MoE block: GpuLayer (gpu.rs:325-541) ---------------------------------------------------------------------- */
/* GpuLayer::upload (gpu.rs:430-449): copies router [E,H], gate_up [E,2I,H], down [E,H,I] (bf16 bits) to the device */
int lastro_layer_create(lastro_ctx *ctx, int32_t experts, int32_t hidden, int32_t inter, int32_t k,
                        const uint16_t *router, const uint16_t *gate_up, const uint16_t *down, lastro_layer **out);
/* GpuLayer::upload for Q8_0 weights (the reference's GpuLayer is bf16 only; its north star adds Q8_0): router [E,H],
 * gate_up [E,2I,H], down [E,H,I] given as rows of 34-byte blocks (fp16 scale, then 32 int8 values; weight = scale *
 * value), repacked on upload into the device row layout; H and I multiples of 32.  forward/add_into/destroy as for
 * bf16 layers. */
int lastro_layer_create_q8_0(lastro_ctx *ctx, int32_t experts, int32_t hidden, int32_t inter, int32_t k,
                             const uint8_t *router, const uint8_t *gate_up, const uint8_t *down, lastro_layer **out);
/* GpuLayer::forward (gpu.rs:461-478): x [H] host in -> y [H] host out, the routing (ids/weights [k], in
 * descending-logit order) and optionally the router logits [E]; any output pointer may be NULL */
int lastro_layer_forward(lastro_layer *layer, const float *x, float *y, int32_t *ids, float *weights,
                         float *logits);
/* GpuLayer::add_into (gpu.rs:480-505): h <- h + resid * moe(xn), xn/h device pointers [H], enqueued on the context's
 * stream without synchronizing; ids/weights (device, [k]) receive the routing when non-NULL */
int lastro_layer_add_into(lastro_layer *layer, const float *xn_dev, float *h_dev, float resid, int32_t *ids_dev,
                          float *weights_dev);
void lastro_layer_destroy(lastro_layer *layer);
/* Allocation-free variant of lastro_layer_forward, with no counterpart in the reference.  For callers that cannot
 * call cudaMalloc -- device memory owned by another runtime's allocator, code running inside a stream capture, or a
 * path where cudaMalloc's implicit synchronisation is not acceptable: they pass every buffer, all device pointers
 * (x [H] f32, router [E,H], gate_up [E,2I,H], down [E,H,I] bf16 bits, outputs y [H] f32, ids [k] i32, weights [k]
 * f32), and the call enqueues the block on `stream` (a cudaStream_t, NULL = legacy stream) of the calling thread's
 * current device without allocating or synchronising.  Its scratch (router logits, a ticket, an error word and the
 * k*I SwiGLU activations) is one file-scope __device__ array of about 66 KB that every GPU loading the library holds
 * until the process exits; limits: experts <= 64, k * inter <= 16384.  The first call on a device looks the array's
 * address up (cudaGetSymbolAddress), so make that first call before any stream capture.  Every call shares the
 * array: calls that overlap on the GPU (other streams, other threads) race; serialise them.  The call clears the
 * array's ticket and error word itself; nothing else in it needs to start at zero.  Returns LASTRO_E_ARG or
 * LASTRO_E_UNSUPPORTED for shapes beyond the limits, before any launch.  The kernels' bounded copy waits report
 * through the scratch's error word: read it with lastro_moe_block_noalloc_status.  The cached scratch address is keyed
 * by device and CUDA context, so a device reset only costs the next call a fresh look-up (again outside a capture). */
int lastro_moe_block_forward_noalloc(const float *x, const uint16_t *router, const uint16_t *gate_up,
                                     const uint16_t *down, int32_t experts, int32_t hidden, int32_t inter, int32_t k,
                                     float *y, int32_t *ids, float *weights, void *stream);
/* Status of the allocation-free block calls on the current device, no counterpart in the reference: enqueues on
 * `stream` a 4-byte copy of the scratch's error word into *status (host or device memory the caller owns; pinned
 * host memory keeps the copy asynchronous), allocating nothing.  After the stream reaches it: 0 when every bounded
 * copy wait of the last call completed, else the code of the wait that gave up (y, ids and weights of that call are
 * then not valid).  Make the first call of either entry point before any stream capture. */
int lastro_moe_block_noalloc_status(int32_t *status, void *stream);

/* ---- whole model: GpuModel (gpu_model.rs:154-455) --------------------------------------------------------------- */
/* GpuModel::upload (gpu_model.rs:191-242): allocates weights, the paged KV cache for max_len positions and the
 * step's scratch; tensors are then loaded with lastro_model_load_tensor or lastro_model_fill_synthetic */
int lastro_model_create(lastro_ctx *ctx, const lastro_model_desc *desc, int32_t max_len, lastro_model **out);
/* copies one checkpoint tensor (model.rs:99-132 names, e.g. "model.layers.3.self_attn.q_proj.weight",
 * "model.layers.3.block_sparse_moe.input_linear.weight"); dtype BF16 (uint16 bits) or F32 (norms only) */
int lastro_model_load_tensor(lastro_model *model, const char *name, int32_t dtype, const int64_t *shape,
                             int32_t ndim, const void *host);
/* random-init every tensor on the device from the synthetic generator (weights ~ std, norms 1 + norm_std) */
int lastro_model_fill_synthetic(lastro_model *model, uint64_t seed, float stddev, float norm_stddev);
/* benchmark/test helper, no reference counterpart: a context of n positions without running n steps.  Every layer's
 * K/V rows of positions [0, n) get synthetic values, element for element the CPU oracle's lo_session_fill_kv (logical
 * element pos * kv_heads * head_dim + head * head_dim + j of layer l's K stream seeded mix64(seed + 2l), of its V
 * stream mix64(seed + 2l + 1); rounded to bf16 in a bf16 cache); the position becomes n */
int lastro_model_fill_kv_synthetic(lastro_model *model, int32_t n, uint64_t seed, float stddev);
/* test helper, no reference counterpart: K and V rows of positions [pos0, pos0 + n) (< the current position) of one
 * layer as f32 [n, kv_heads * head_dim] (bf16 caches widened exactly); either output may be NULL */
int lastro_model_read_kv(lastro_model *model, int32_t layer, int32_t pos0, int32_t n, float *k_out, float *v_out);
/* GpuModel::step (gpu_model.rs:251-267): one token; logits [V] (already / logits_scaling), the greedy next token
 * (argmax, last maximum on ties), routes ids/weights [layers*k]; every output may be NULL */
int lastro_model_step(lastro_model *model, int32_t token, float *logits, int32_t *next_token, int32_t *route_ids,
                      float *route_weights);
/* greedy loop of bin/m1b-gulosa.rs:84-110 kept on the device: feeds prompt[0..n_prompt) then generates n_new
 * tokens, each step's argmax fed back without a host round trip; out_ids [n_new] may be NULL */
int lastro_model_generate(lastro_model *model, const int32_t *prompt, int32_t n_prompt, int32_t n_new,
                          int32_t *out_ids);
/* the greedy loop of geracao_regra.rs:181-245 in normal use: feeds prompt[0..n_prompt), then generates up to n_new
 * tokens, each fed back on the device, stopping after the first `eos` (Granite's <|end_of_text|> is id 0,
 * geracao_regra.rs:31; eos < 0 never stops, which is lastro_model_generate).  out_ids [n_new] receives the generated
 * ids, the end-of-text token included; *n_out their count.  The model ends where the reference's loop leaves it: the
 * prompt and every generated token but the last have been fed (the steps run in chunks of 16 with one host read each,
 * and the position is rolled back over any step run past the end of text). */
int lastro_model_generate_until(lastro_model *model, const int32_t *prompt, int32_t n_prompt, int32_t n_new,
                                int32_t eos, int32_t *out_ids, int32_t *n_out);
/* device-resident greedy decode of n tokens continuing from the last token (no host copies; for timing) */
int lastro_model_decode(lastro_model *model, int32_t n);
/* the multi-position step (cuda_backend.rs:264-274, cpu.rs:234-297 experts_step): n consecutive positions of the
 * model's sequence (1 <= n <= 32) in one step, causal inside the step (position i attends to every earlier position
 * and itself), on the batched path's tensor-core GEMMs (bf16 weights).  Per-position results equal the token-by-token
 * step up to summation order.  logits [n, V] (/ logits_scaling) and next [n] (greedy ids, last maximum) may be NULL;
 * the position advances by n and the last position's greedy id becomes the token a device-side decode continues
 * from.  Allocates its step scratch on first use. */
int lastro_model_step_positions(lastro_model *model, int32_t n, const int32_t *tokens, float *logits, int32_t *next);
/* GpuModel::reset (gpu_model.rs:244-247): position 0, page table reset */
int lastro_model_reset(lastro_model *model);
int lastro_model_position(const lastro_model *model, int32_t *pos);
/* per-kernel device time of `steps` decode steps (direct launches with an event between kernels, no graph, no
 * PDL), averaged per step and summed over layers: kernel_ms[0..8] = qkv_rope, attention, oproj, router, gate_up,
 * down, head, fused_step (the whole step when the fused kernel runs it; then the others are 0), moe (the one-launch
 * MoE block; then gate_up and down are 0).  Advances the
 * position like lastro_model_decode.  No reference counterpart: measurement only (the reference's step_probe,
 * gpu_model.rs:275-300, times whole steps). */
int lastro_model_profile(lastro_model *model, int32_t steps, float *kernel_ms, int32_t n_kinds);
/* in-graph timeline of `steps` decode steps: the step graph captured again with every CTA stamping the global timer
 * (start, release from griddepcontrol.wait, exit) and replayed like lastro_model_decode.  Per kernel kind (the kinds of
 * lastro_model_profile), summed over layers and averaged over steps: exposed_ms = the kind's share of the step's
 * critical path (each launch's last exit minus the previous launch's, so the kinds sum to the step), span_ms = last
 * exit minus first CTA start (includes the time resident under the predecessor), wait_ms = first release from
 * griddepcontrol.wait minus the previous launch's last exit (the hand-off latency); step_ms = first start to last exit.  Launches without stamps (tensor-core attention) count 0.  Advances the
 * position like lastro_model_decode.  No reference counterpart: measurement only. */
int lastro_model_trace(lastro_model *model, int32_t steps, float *exposed_ms, float *span_ms, float *wait_ms,
                       int32_t n_kinds, float *step_ms);
/* the stamps of launch `launch` (in step order) of the last step lastro_model_trace timed: for each of up to 1024
 * CTAs, LASTRO_TRACE_WORDS words: global-timer ns of start, release from griddepcontrol.wait and exit, then 8 of the
 * kernel's own milestones (0 where not stamped); words >= 1024 * LASTRO_TRACE_WORDS.  Diagnostics only. */
#define LASTRO_TRACE_WORDS 11
int lastro_model_trace_raw(const lastro_model *model, int32_t launch, unsigned long long *out, int32_t words);
/* tuning: use CUDA graphs (default 1), programmatic dependent launch between the per-layer kernels (default 1),
 * and the fused step -- the whole step as one persistent cooperative launch, one CTA per SM -- where the model's
 * shapes fit it (default 0: on B200 it measures slower than the per-layer kernels; lastro_model_fused reports
 * whether the fused step runs) */
int lastro_model_set_options(lastro_model *model, int32_t use_graphs, int32_t use_pdl, int32_t use_fused);
/* the MoE block of every layer as one persistent launch (1: routing, gate_up and down streamed through one ring of
 * shared memory, a grid barrier between them) or as the gate_up and down kernels (0, the default: faster on C3);
 * LASTRO_E_UNSUPPORTED for 1 when the shapes do not fit it */
int lastro_model_set_moe(lastro_model *model, int32_t one_launch);
/* tuning of the batch-1 attention kernel (CUDA-core, the default): attn_splits context splits per KV head (8 or 16;
 * 0 picks 8 when a split's rows fit one pass of the CTA, else 16) and how the splits are merged (0: by the last CTA
 * of each KV head, through global memory, the default; 1: by the output projection as it loads the attention output;
 * 2: the splits of a KV head are one thread-block cluster that merges them in distributed shared memory);
 * flags: LASTRO_TUNE_OPROJ_SMEM stages the output projection's weight rows in shared memory in 256-thread CTAs
 * (else they sit in the registers of 512-thread CTAs); LASTRO_TUNE_PREFETCH_DOWN has the gate_up kernel hint the
 * chosen experts' down rows into L2; LASTRO_TUNE_ATTN_TMA stages bf16 K/V rows as 8-row TMA boxes with the 128-byte
 * swizzle, whose reads are free of shared-memory bank conflicts (else one bulk copy per page run, the default);
 * LASTRO_TUNE_SPEC_L2 fetches the experts predicted from the layer's input early (bf16 weights: the qkv kernel
 * computes the router logits of the layer's input, the top-k of which the output projection's CTAs hint into L2 while
 * the attention runs); LASTRO_TUNE_SPEC_STAGE instead has each gate_up CTA stream the rows of the expert predicted for
 * its slot into shared memory before the routing is known (experts the prediction missed are staged after it);
 * LASTRO_TUNE_SPEC_ATTN hints the predicted experts' gate_up and down weights into L2 from the attention kernel's
 * CTAs, a share each, as soon as the qkv kernel has taken their top-k.  All three are off by default.  LASTRO_TUNE_ATTN_MMA scores and sums bf16 K/V
 * on tensor cores (mma.sync with q and the probabilities split into bf16 hi + lo, a relative residue below 2^-16)
 * instead of f32 CUDA-core dots.  LASTRO_TUNE_DOWN_ROUTES has every down CTA reduce the router shares itself instead
 * of taking the routing gate_up's first CTA publishes (a flag per layer stamped with a step counter, a bounded wait
 * that falls back to the reduction).  The cluster merge (attn_merge 2) runs without the TMA and tensor-core forms.
 * Results are bitwise the same for every flag but LASTRO_TUNE_ATTN_MMA; LASTRO_E_UNSUPPORTED for the TMA or
 * tensor-core form with f32 KV. */
#define LASTRO_TUNE_OPROJ_SMEM 1
#define LASTRO_TUNE_PREFETCH_DOWN 2
#define LASTRO_TUNE_ATTN_TMA 4
#define LASTRO_TUNE_SPEC_L2 8
#define LASTRO_TUNE_SPEC_STAGE 16
#define LASTRO_TUNE_ATTN_MMA 32
#define LASTRO_TUNE_DOWN_ROUTES 64
#define LASTRO_TUNE_SPEC_ATTN 128
int lastro_model_set_tuning(lastro_model *model, int32_t attn_splits, int32_t attn_merge, int32_t flags);
/* 1 when the MoE blocks run as one launch per layer */
int lastro_model_moe(const lastro_model *model);
/* 1 when decode steps run as the fused step kernel (shapes fit and the option is on), else 0 */
int lastro_model_fused(const lastro_model *model);
/* attention kernel of the step chain with bf16 KV: tensor cores with TMA page loads (1) or the CUDA-core split kernel
 * (0, the default: faster at batch 1 on B200; the only one with f32 KV) */
int lastro_model_set_attention(lastro_model *model, int32_t tensor_cores);
void lastro_model_destroy(lastro_model *model);

/* ---- checkpoints on disk: safetensors + config.json (weights.rs:52-122, model.rs:34-61, model.rs:99-132) ------- */
/* Host-only (no GPU needed) except lastro_model_load_checkpoint.  Errors of the checkpoint and config calls are
 * written to err (err_len bytes, may be NULL) like the reference's WeightError / Config::from_json strings:
 * LASTRO_E_ARG for a malformed file or a refusal, LASTRO_E_IO for a file that cannot be opened or read,
 * LASTRO_E_UNSUPPORTED for a config the kernels do not implement. */
typedef struct lastro_checkpoint lastro_checkpoint;
/* Checkpoint::open (weights.rs:52-106): indexes every *.safetensors file of dir (sorted by name): header length
 * (8 bytes little-endian, at most 100 MiB), JSON header name -> {dtype, shape, data_offsets}; refuses missing fields,
 * non-numeric or != 2 data_offsets, offsets that overflow or end past the file.  Only the index stays in memory. */
int lastro_checkpoint_open(const char *dir, lastro_checkpoint **out, char *err, int32_t err_len);
void lastro_checkpoint_close(lastro_checkpoint *ck);
/* number of tensors indexed */
int lastro_checkpoint_count(const lastro_checkpoint *ck);
/* one index entry: dtype string (dtype_len bytes), shape (up to max_ndim dims; -1 for a dim beyond INT64_MAX) and
 * its rank; LASTRO_E_ARG when the tensor is absent */
int lastro_checkpoint_tensor(const lastro_checkpoint *ck, const char *name, char *dtype, int32_t dtype_len,
                             int64_t *shape, int32_t max_ndim, int32_t *ndim);
/* Checkpoint::bf16 (weights.rs:108-122): a whole BF16 tensor into dst (capacity elements); refuses an absent tensor,
 * another dtype, or a byte count that does not match the shape (overflow included) */
int lastro_checkpoint_read_bf16(const lastro_checkpoint *ck, const char *name, uint16_t *dst, int64_t capacity,
                                char *err, int32_t err_len);
/* Config::from_json (model.rs:34-61) on the text of a config.json: refuses model_type != "granitemoe", a non-null
 * rope_scaling, attention_bias true and tie_word_embeddings false (LASTRO_E_UNSUPPORTED), or a missing field
 * (LASTRO_E_ARG); head_dim defaults to hidden / heads.  weight_dtype and kv_dtype come back BF16. */
int lastro_config_from_json(const char *json, lastro_model_desc *out, char *err, int32_t err_len);
/* the same on the checkpoint directory's config.json */
int lastro_checkpoint_config(const lastro_checkpoint *ck, lastro_model_desc *out, char *err, int32_t err_len);
/* HostModel::load + GpuModel::upload (model.rs:99-132, block.rs:31-53): every tensor of the model, each refused
 * before it is read when absent or of another shape, dtype or byte size; BF16 tensors, or for a Q8_0 model its linear
 * weights as U8 tensors whose last axis holds each row's 34-byte blocks.  Errors through lastro_last_error. */
int lastro_model_load_checkpoint(lastro_model *model, const lastro_checkpoint *ck);

/* ---- batched decode with expert parallelism (no counterpart in the reference, which decodes one sequence) ------- */
/* Many independent sequences decoded together on a model's weights (bf16); each sequence's results equal its own
 * single-sequence step up to summation order (the reference's multi-position contract, cpu.rs:234-238).  The MoE
 * experts are partitioned over the `world` ranks of an expert-parallel group, one process per GPU: rank r computes
 * E/world experts (by default [r*E/world, (r+1)*E/world); lastro_batch_set_expert_placement) for the pairs every rank
 * routes to them, while attention and the dense layers stay with each rank's own sequences.  Every rank creates its batch with the same max_seqs and world, passes the handle
 * of its exchange region (lastro_batch_exchange_handle, 64 bytes) to the others, and connects with all of them in rank
 * order (lastro_batch_connect; world 1: handles may be NULL).  The ranks then call lastro_batch_step/decode the same
 * number of times, each with at least one of its own sequences.  Destroy a batch before its model.  A rank that does
 * not arrive makes the others' waits give up after 10 s (LASTRO_E_CUDA, batch poisoned; lastro_batch_set_wait_limit). */
typedef struct lastro_batch lastro_batch;
int lastro_batch_create(lastro_model *model, int32_t max_seqs, int32_t max_len, int32_t rank, int32_t world,
                        lastro_batch **out);
int lastro_batch_exchange_handle(lastro_batch *batch, void *handle, int32_t bytes);
int lastro_batch_connect(lastro_batch *batch, const void *handles, int32_t bytes_each);
/* per-layer router logit bias [layers, experts] added before the top-k (NULL removes it): a workload knob for skewed
 * expert load; Granite's router has no bias */
int lastro_batch_set_router_bias(lastro_batch *batch, const float *bias);
/* owner[e] (n_experts = E entries): the rank that computes expert e, every rank owning E/world experts.  All ranks of
 * the group set the same placement between the same two steps; results do not depend on it (each expert still sees
 * its pairs in global token order).  Refused (batch usable) for a wrong count or an uneven placement. */
int lastro_batch_set_expert_placement(lastro_batch *batch, const int32_t *owner, int32_t n_experts);
/* one token for each of n distinct sequences (ids < max_seqs): next [n] greedy ids (last maximum), logits [n, V] and
 * route_ids [n, layers, k] when non-NULL */
int lastro_batch_step(lastro_batch *batch, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t *next,
                      float *logits, int32_t *route_ids);
/* `steps` greedy steps of the n sequences on the device, each step's ids fed back as the next step's tokens;
 * out_ids [steps, n] when non-NULL */
int lastro_batch_decode(lastro_batch *batch, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t steps,
                        int32_t *out_ids);
/* a context of n positions with synthetic K/V for sequence `seq` (benchmarks and profiling) */
int lastro_batch_fill_kv_synthetic(lastro_batch *batch, int32_t seq, int32_t n, uint64_t seed, float stddev);
int lastro_batch_reset(lastro_batch *batch, int32_t seq);
int lastro_batch_position(const lastro_batch *batch, int32_t seq, int32_t *pos);
/* mean device ms per step of each kernel kind over `steps` directly launched greedy steps (tokens as for
 * lastro_batch_decode), timed with events between launches: norm (layer 0), qkv, rope_kv, attention, oproj, router
 * (with the dispatch and the grouping of the received pairs), group (0: part of the router), gate_up, down (with the
 * return), combine (with the next norm), lm_head, argmax (n_kinds >= 12) */
int lastro_batch_profile(lastro_batch *batch, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t steps,
                         float *kernel_ms, int32_t n_kinds);
/* in-graph timeline of `steps` graph-replayed steps (tokens as for lastro_batch_decode; the positions advance):
 * every CTA of the step's launches stamps the global timer (start, release from griddepcontrol.wait, exit); per kernel
 * kind (lastro_batch_profile's order) the ms per step of its share of the step's critical path (exposed; they sum to
 * the step), first CTA start to last CTA exit summed over the launches (span), and the hand-off from the previous
 * launch's last exit to its first release (wait); step_ms first start to last exit.  All ranks of a group call it
 * together.  Diagnostics only; no reference counterpart. */
int lastro_batch_trace(lastro_batch *batch, int32_t n, const int32_t *seq_ids, const int32_t *tokens, int32_t steps,
                       float *exposed_ms, float *span_ms, float *wait_ms, int32_t n_kinds, float *step_ms);
/* the stamps of launch `launch` (0 the layer-0 norm, then 8 per layer: qkv, rope_kv, attention, oproj, router, gate_up,
 * down, combine; then lm_head, argmax) of the last step lastro_batch_trace timed, laid out as for
 * lastro_model_trace_raw.  Milestones: the router 5 (RMSNorm done), 0 (router logits), 3 (top-k), 4 (MoE rows sent),
 * 1 (expert ids sent) and, in its last CTA, 2 (dispatch flag published; the exit then ends the wait for the senders
 * and the grouping); the combine 0 (every owner's return flag seen); the tcgen05 GEMMs 0 (set up), 1, 4 and 5 (the
 * first, second and middle stage landed), 2 (last MMAs issued), 3 (accumulator complete) */
int lastro_batch_trace_raw(const lastro_batch *batch, int32_t launch, unsigned long long *out, int32_t words);
/* use_graphs: replay each step as a CUDA graph (default 1); use_tcgen05: the GEMMs on the 5th-generation tensor cores
 * with tensor-memory accumulators, warp-specialised with TMA weight tiles (2, default), the same with all threads
 * loading the stages (1), or on mma.sync with register accumulators (0); attn_tc: attention on tensor cores with TMA
 * page loads (1, the default with bf16 KV) or on CUDA cores (0, the only choice with f32 KV) */
int lastro_batch_set_options(lastro_batch *batch, int32_t use_graphs, int32_t use_tcgen05, int32_t attn_tc);
/* bound of every wait on another rank's exchange flag (default 10 s; 1 ms to 600 s): a rank that does not arrive
 * within it makes the step return LASTRO_E_CUDA and poisons the batch; later waits of the same step give up at once
 * (gpu_model.rs:249-267's poison policy; no reference counterpart for the limit itself) */
int lastro_batch_set_wait_limit(lastro_batch *batch, uint64_t wait_ns);
void lastro_batch_destroy(lastro_batch *batch);

/* ---- text I/O: byte-level BPE tokenizer and the Granite 3.1 chat template (rust/moe-rt/src/tokenizador.rs) ----
 * Host-only.  Replaces Tokenizador (tokenizador.rs:192-467), renderiza_chat (:512-541) and formata_data (:544-561).
 * Errors: LASTRO_E_ARG for bad arguments, text that is not UTF-8, an id outside the vocabulary, or an output buffer
 * too small (the needed size is still written to the count argument); LASTRO_E_IO for a file that cannot be read;
 * LASTRO_E_UNSUPPORTED for a tokenizer.json outside the Granite configuration (ErroTokenizador::Formato: normalizer,
 * pre-tokenizer other than ByteLevel{add_prefix_space false, use_regex true}, decoder, dropout, unk token, byte
 * fallback, subword affixes, ignore_merges, added tokens with lstrip/rstrip/single_word/normalized, sparse ids, merges
 * outside the vocabulary); err (errlen bytes, NUL-terminated) receives a message. */
typedef struct lastro_tokenizer lastro_tokenizer;
/* Tokenizador::carrega (tokenizador.rs:215-218) */
int lastro_tokenizer_load(const char *path, lastro_tokenizer **out, char *err, int32_t errlen);
/* Tokenizador::de_bytes (tokenizador.rs:221-345): from the tokenizer.json text */
int lastro_tokenizer_from_json(const char *json, size_t len, lastro_tokenizer **out, char *err, int32_t errlen);
void lastro_tokenizer_destroy(lastro_tokenizer *tok);
/* largest id + 1 (tamanho_vocabulario, tokenizador.rs:347-349) */
int32_t lastro_tokenizer_vocab_size(const lastro_tokenizer *tok);
/* codifica (tokenizador.rs:420-448): UTF-8 text of len bytes -> ids, as `tokenizers` encodes it without special
 * tokens added (no BOS); *n_ids = the count (also when cap is too small) */
int lastro_tokenizer_encode(const lastro_tokenizer *tok, const char *text, size_t len, int32_t *ids, int32_t cap,
                            int32_t *n_ids);
/* decodifica_bytes (tokenizador.rs:451-460): the exact bytes; added tokens as their literal text */
int lastro_tokenizer_decode_bytes(const lastro_tokenizer *tok, const int32_t *ids, int32_t n, char *out, size_t cap,
                                  size_t *n_out);
/* decodifica (tokenizador.rs:463-466): the bytes as UTF-8 text, each maximal invalid subsequence of the whole sequence
 * replaced by U+FFFD (no clean-up of spaces before punctuation) */
int lastro_tokenizer_decode(const lastro_tokenizer *tok, const int32_t *ids, int32_t n, char *out, size_t cap,
                            size_t *n_out);
/* pre_tokeniza (tokenizador.rs:125-177): the GPT-2 regex pieces of UTF-8 text, as the byte offset where each ends */
int lastro_tokenizer_pretokenize(const char *text, size_t len, int32_t *ends, int32_t cap, int32_t *n_pieces);
#define LASTRO_ROLE_SYSTEM 0
#define LASTRO_ROLE_USER 1
#define LASTRO_ROLE_ASSISTANT 2
/* renderiza_chat (tokenizador.rs:512-541): the Granite 3.1 chat template for n >= 1 messages (roles LASTRO_ROLE_*,
 * contents of lens bytes); a first system message is the system turn, else the default one with `date`
 * (strftime("%B %d, %Y"), see lastro_format_date); add_generation_prompt opens an assistant turn after the last
 * message that follows the system turn.  *n_out = the rendered length (also when cap is too small). */
int lastro_chat_render(const int32_t *roles, const char *const *contents, const size_t *lens, int32_t n,
                       int32_t add_generation_prompt, const char *date, char *out, size_t cap, size_t *n_out);
/* formata_data (tokenizador.rs:544-561): "November 07, 2026"; LASTRO_E_ARG for an invalid date (years 1..9999) */
int lastro_format_date(int32_t year, int32_t month, int32_t day, char *out, int32_t cap);

#ifdef __cplusplus
}
#endif
#endif
