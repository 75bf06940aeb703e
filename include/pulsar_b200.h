/*
 * pulsar_b200 - C ABI of the B200-native (sm_100a) Pulsar-283M KV-cache decode engine.
 *
 * Conventions
 *   - Every entry point returns an int status: PULSAR_OK (0) or a negative PULSAR_ERR_*;
 *     pulsar_last_error() returns a message for the calling thread's last failure.
 *   - Pointers named *_dev are device pointers; *_host are host pointers. `stream` is a
 *     cudaStream_t passed as void* (NULL = the legacy default stream). Every kernel is
 *     launched on that stream and every launch is checked.
 *   - No torch types cross this boundary: plain pointers, sizes and strides.
 *   - Ops (pulsar_op_*) are functional: the caller owns and sizes every output buffer.
 *     Engine calls (pulsar_engine_*) use memory the engine allocated at create time; the
 *     token path allocates nothing.
 *   - An engine handle is not thread-safe: one host thread drives one engine.
 */
#ifndef PULSAR_B200_H
#define PULSAR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PULSAR_OK 0
#define PULSAR_ERR_INVALID (-1)     /* bad argument, shape or dtype */
#define PULSAR_ERR_CUDA (-2)        /* CUDA runtime / launch error */
#define PULSAR_ERR_OOM (-3)         /* device allocation failed */
#define PULSAR_ERR_STATE (-4)       /* call not valid in the engine's current state */
#define PULSAR_ERR_UNSUPPORTED (-5) /* configuration the compiled kernels do not cover */
#define PULSAR_ERR_CAPACITY (-6)    /* KV / row capacity exceeded */

/* Message of the calling thread's last failed call ("" if none). */
const char* pulsar_last_error(void);
/* ABI version (major * 10000 + minor * 100 + patch). */
int pulsar_abi_version(void);

/* ==================================================================================
 * pulsar_cuda forward ops. Each replaces one binding of the reference extension
 * (csrc/pulsar_cuda.cpp:199-279) and keeps its argument meaning; the reference checks
 * (TORCH_CHECK) become PULSAR_ERR_INVALID with the same message text.
 * ================================================================================== */

/* csrc/kernels.cu:224-266 rmsnorm_forward_cuda (binding csrc/pulsar_cuda.cpp:200).
 * x [rows, D] bf16, weight [D] f32 -> y [rows, D] bf16, rsqrt [rows] f32. */
int pulsar_op_rmsnorm(const void* x_dev, const float* weight_dev, int64_t rows, int64_t D, float eps,
                      void* y_dev, float* rsqrt_dev, void* stream);

/* csrc/kernels.cu:908-965 rope_forward_cuda (binding :206). qk [rows, Dh] bf16 where the
 * position of row r is r % T; cos/sin [T, Dh/2] f32 -> y [rows, Dh] bf16. */
int pulsar_op_rope(const void* qk_dev, const float* cos_dev, const float* sin_dev, int64_t rows, int64_t T,
                   int64_t Dh, void* y_dev, void* stream);

/* csrc/kernels.cu:825-863 fused_swiglu_forward_cuda (binding :204). gu [rows, 2*d_ff] bf16
 * -> out [rows, d_ff] bf16, out = silu(gate) * up computed in fp32. */
int pulsar_op_swiglu(const void* gu_dev, int64_t rows, int64_t d_ff, void* out_dev, void* stream);

/* csrc/kernels.cu:2417-2491 moe_router_topk_forward_cuda (binding :244-255).
 * logits [N, E] (f32, or bf16 when logits_bf16 != 0), expert_bias [E] f32; E <= 32,
 * 1 <= K <= min(8, E). Outputs: topk_idx [N, K] i64, topk_weights [N, K] bf16,
 * z_loss [1] f32 (z_loss_weight * mean_t lse_t^2 over centred logits; 0 when
 * z_loss_weight <= 0), probs_mean [E] f32 (mean sigmoid score).
 * workspace_dev: N * (E + 1) floats of caller scratch (deterministic two-pass means). */
int pulsar_op_moe_router_topk(const void* logits_dev, int logits_bf16, const float* expert_bias_dev,
                              int64_t N, int64_t E, int64_t K, float z_loss_weight, int64_t* topk_idx_dev,
                              void* topk_weights_dev, float* z_loss_dev, float* probs_mean_dev,
                              float* workspace_dev, void* stream);

/* No counterpart in the reference. The router top-k above without a caller workspace, for
 * callers that cannot allocate device memory (a host whose memory manager owns every
 * device byte, or a foreign-language caller without a device allocator): the scratch is a
 * 4 MiB array compiled into the library, present on every GPU that loads it until exit.
 * Limit: N * (E + 1) <= 1,048,576 floats, else PULSAR_ERR_CAPACITY. Allocates nothing.
 * The first call on each device looks up the array's device address (with that device
 * current); make that first call before any stream capture begins. The address is looked up
 * again when the calling thread's current context is not the one it was found in (after
 * cudaDeviceReset, for instance); make the first call after such a reset before any stream
 * capture too. All calls share the
 * array: calls whose executions overlap on the GPU (for example on two streams) race.
 * Nothing in it has to start at zero: each call writes every element it reads. */
int pulsar_op_moe_router_topk_noalloc(const void* logits_dev, int logits_bf16, const float* expert_bias_dev,
                                      int64_t N, int64_t E, int64_t K, float z_loss_weight,
                                      int64_t* topk_idx_dev, void* topk_weights_dev, float* z_loss_dev,
                                      float* probs_mean_dev, void* stream);

/* csrc/kernels.cu:2716-2765 qk_rmsnorm_rope_forward_cuda (binding :229-230).
 * x: n_vec vectors of 64 bf16 with element strides (sB, sH, sT) over the logical
 * [B, n_heads, T, 64] index, vector v = ((b * n_heads) + h) * T + t; weight [n_heads, 64]
 * f32; cos/sin [T, 32] f32. Outputs y [n_vec, 64] bf16 contiguous, rsqrt [n_vec] f32. */
int pulsar_op_qk_rmsnorm_rope(const void* x_dev, int64_t sB, int64_t sH, int64_t sT, int64_t n_vec,
                              int64_t n_heads, int64_t T, const float* weight_dev, const float* cos_dev,
                              const float* sin_dev, float eps, void* y_dev, float* rsqrt_dev, void* stream);

/* csrc/kernels.cu:2844-2877, 2930-2958 fused_attn_gate_forward_cuda (binding :233-234).
 * attn [B, H, T, 64] bf16 contiguous, gate_logits [B, T, H] f32 -> out [B, T, H*64] bf16. */
int pulsar_op_attn_gate(const void* attn_dev, const float* gate_logits_dev, int64_t B, int64_t H, int64_t T,
                        void* out_dev, void* stream);

/* csrc/kernels.cu:3653-3691 causal_depthwise_conv1d_k4_forward_cuda (binding :271-273).
 * x [B, T, D] bf16, weight [D, 4] f32 -> y[b,t,d] = x + sum_k w[d,k] * x[b,t-k,d]. */
int pulsar_op_conv1d_k4(const void* x_dev, const float* weight_dev, int64_t B, int64_t T, int64_t D,
                        void* y_dev, void* stream);

/* csrc/kernels.cu:1633-1664 moe_combine_forward_cuda (binding :214-216).
 * expert_outputs [E, C, D] bf16, topk_idx [N, K] i64, topk_weights [N, K] bf16,
 * token_to_slot [N, K] i32 (-1 dropped), shared_out [N, D] bf16 or NULL -> out [N, D] bf16. */
int pulsar_op_moe_combine(const void* expert_outputs_dev, const int64_t* topk_idx_dev,
                          const void* topk_weights_dev, const int32_t* token_to_slot_dev,
                          const void* shared_out_dev, int64_t N, int64_t K, int64_t E, int64_t C, int64_t D,
                          void* out_dev, void* stream);

/* csrc/kernels.cu:1548-1605 moe_dispatch_forward_cuda (binding :209-211).
 * x [N, D] bf16 -> expert_inputs [E, C, D] bf16; unused slots are zeroed (all of them, or
 * only the tail past expert_counts[e] when expert_counts_dev [E] i64 is given). */
int pulsar_op_moe_dispatch(const void* x_dev, const int64_t* topk_idx_dev, const int32_t* token_to_slot_dev,
                           const int64_t* expert_counts_dev, int64_t N, int64_t K, int64_t E, int64_t C,
                           int64_t D, void* expert_inputs_dev, void* stream);

/* ==================================================================================
 * Engine: the KV-cache decode path of src/infer.py on the device.
 * ================================================================================== */

typedef struct pulsar_engine pulsar_engine;

typedef struct {
    int32_t vocab_size;        /* multiple of 256 */
    int32_t max_pulses;        /* leading dim of per-pulse parameters (reference: 8) */
    int32_t loop_lora_rank;    /* 0 = no loop adapters */
    float loop_lora_alpha;
    float rms_eps;
    float logit_softcap;       /* <= 0: no softcap */
    int32_t base_seq_len;      /* YaRN base (1024) */
    int32_t use_canon_conv;
    int32_t per_pulse_bias;
    int32_t max_batch;         /* sequence slots, 1..1024 */
    int32_t max_seq_len;       /* KV positions per slot (prompt + generated + slack) */
    int32_t max_prefill;       /* longest prompt one prefill call accepts */
    int32_t kv_fp32;           /* 0: bf16 KV cache (default); 1: fp32 KV cache (parity mode) */
    int32_t device;            /* CUDA device ordinal */
} pulsar_engine_config;

/* Replaces PulsarInferenceEngine.__init__ + load_inference_model (src/infer.py:184-209,
 * 785-817): allocates the weight arena, the per-slot KV cache and the workspaces. */
int pulsar_engine_create(const pulsar_engine_config* cfg, pulsar_engine** out);
int pulsar_engine_destroy(pulsar_engine* eng);

/* Upload one reference state_dict tensor (name as in PulsarForCausalLM.state_dict(),
 * fp32 host data, row-major, numel checked). rope inv_freq tables are passed as
 * "rope_local.inv_freq" / "rope_global.inv_freq" [32]. */
int pulsar_engine_set_tensor(pulsar_engine* eng, const char* name, const float* data_host, int64_t numel);

/* Build the per-pulse bf16 arena: loop-adapter merges (src/model.py:716-727), expert
 * transposes, rope tables. Required once after all set_tensor calls. */
int pulsar_engine_finalize(pulsar_engine* eng);

/* Bytes of the device weight arena / KV cache / workspaces. */
int pulsar_engine_memory(const pulsar_engine* eng, int64_t* arena_bytes, int64_t* kv_bytes, int64_t* work_bytes);

/* PulsarInferenceEngine.prefill (src/infer.py:353-461) for one sequence slot.
 * ids_dev [T] i32. Writes last-position logits [V] f32 (no softcap, as the reference)
 * and sets the slot length to T. */
int pulsar_engine_prefill(pulsar_engine* eng, int32_t slot, const int32_t* ids_dev, int32_t T, float* logits_dev,
                          void* stream);

/* PulsarForCausalLM.forward with labels=None (src/model.py:1956-2125), the full-sequence pass
 * that model.generate (src/model.py:2246-2317) recomputes for every new token: ids [T] (device
 * int32) -> the last position's softcapped logits [V] (device fp32). It differs from
 * pulsar_engine_prefill in the reference's own ways: the value residual of layer 0 / pulse 0
 * carries into every pulse, global layers scale queries by 1 + 0.1 ln(max(t + 1, 1024) / 1024),
 * local layers attend causally over the whole sequence (the reference switches to its sliding
 * window only beyond 4096 tokens), and the logits are softcapped. T <= min(max_prefill, 2048)
 * (the local layers' ring holds every key); PULSAR_ERR_CAPACITY beyond. Uses the slot's cache
 * as scratch and leaves the slot empty (length 0). */
int pulsar_engine_forward(pulsar_engine* eng, int32_t slot, const int32_t* ids, int32_t T, float* logits,
                          void* stream);

/* decode_pulse_pass (src/infer.py:463-524) over R rows, 1 <= R <= max(32, 8 * max_batch)
 * (option "wide_rows"). R <= 5: one persistent kernel; R <= 32: per-op GEMV kernels; more
 * rows (or option "wide" = 1): tiled GEMMs over all rows with the routed experts grouped
 * per expert.
 * rows_dev [R] x int4 {slot, pos, token, 0} (the last field is reserved: bit 0 marks a row
 * that exited early inside generate_greedy and must be 0 here). Rows of the same slot must have
 * consecutive positions (block-verify: a row sees in-block predecessors' K/V of this
 * pulse). h_prev_dev / h0n_dev [R, 1024] f32 (ignored for pulse 0). Outputs h_out,
 * h0n_out [R, 1024] f32; logits [R, V] f32 (softcapped) unless logits_dev is NULL. */
int pulsar_engine_pulse(pulsar_engine* eng, int32_t pulse, int32_t R, const int32_t* rows_dev,
                        const float* h_prev_dev, const float* h0n_dev, float* h_out_dev, float* h0n_out_dev,
                        float* logits_dev, void* stream);

/* Sequence-slot KV length (UnifiedKVCache.seq_len / checkpoint_state / restore_state,
 * src/infer.py:99, 159-168). Restoring a shorter length is the rollback. */
int pulsar_engine_get_length(pulsar_engine* eng, int32_t slot, int32_t* length);
int pulsar_engine_set_length(pulsar_engine* eng, int32_t slot, int32_t length);

/* Read cached keys / values (UnifiedKVCache.layers[layer]["k"], ["v"] of the reference,
 * src/infer.py:86-96, which scripts/benchmark.py:411-417 reads): positions [pos0, pos0 + n)
 * of one slot and layer, every kv head, as fp32 [4][n][64] into k_host and v_host (converted
 * from bf16 when the cache is bf16). Local layers keep a ring of their last 2048 positions:
 * a position older than that reads whatever later position shares its ring entry. Waits for
 * the device; not for the token path (it allocates a staging buffer). */
int pulsar_engine_read_kv(pulsar_engine* eng, int32_t slot, int32_t layer, int32_t pos0, int32_t n, float* k_host,
                          float* v_host);

/* The attention step of pulsar_engine_prefill for one layer (src/infer.py:422-435 masks: causal,
 * and for local layers with T > 1024 the truncated cache of the last 1024 positions with the
 * causal mask aligned top-left), over the slot's cached keys and values of positions 0..T-1,
 * which a prefill of T tokens wrote. q_dev: [T][16][64] fp32 normed and rotated queries
 * (unscaled); out_dev: [T][16][64] fp32. tensor_cores 1: the tcgen05 kernel that prefill uses,
 * 0: the fp32 SIMT kernel (the engine option "tc_attn" selects between them inside prefill).
 * Device pointers; enqueued on `stream`. */
int pulsar_engine_prefill_attention(pulsar_engine* eng, int32_t slot, int32_t layer, int32_t T, const float* q_dev,
                                    float* out_dev, int32_t tensor_cores, void* stream);

/* The decode attention of the per-op and many-row pulse passes for one layer (src/infer.py
 * 290-306 per row: softmax(q k^T / 8) v, without the head gate), over the keys the slot holds
 * at positions 0..pos (the last 1024 of them on a local layer). rows_dev: [R][4] int32 (slot,
 * pos, unused, unused), 16-byte aligned, runs of consecutive positions of one slot forming
 * verify blocks of up to rows_per_block (1..8) rows; q_dev: [R][16][64] fp32 normed and rotated
 * queries (unscaled); out_dev: [R][16][64] fp32 (0 for a row with no visible key or an invalid
 * slot or position). tensor_cores 1: k_attn_dec_tc (bf16 cache only; an fp32 cache takes the
 * SIMT kernel either way), 0: the SIMT k_attn_flash. Device pointers; enqueued on `stream` and
 * waited for (it allocates its partial buffer): a check, not for the token path. */
int pulsar_engine_decode_attention(pulsar_engine* eng, int32_t layer, int32_t R, const int32_t* rows_dev,
                                   int32_t rows_per_block, const float* q_dev, float* out_dev, int32_t tensor_cores,
                                   void* stream);

/* Greedy decode loop, reference semantics (stream_generate with temperature 0 and
 * repetition_penalty 1, src/infer.py:551-621): starting from the prefill logits already
 * in the slot's state, emit n_new tokens. gamma == 0: exact sequential decode (3 pulses
 * per token). gamma >= 1: draft gamma tokens from the pulse-1 exit, verify the gamma+1
 * block with pulses 2-3 in one batched pass, accept while argmax agrees, roll back.
 * 1 <= n_seq <= max_batch, 0 <= gamma <= 7, distinct slots.
 * Runs device-resident (CUDA graphs, no per-token host sync).
 * first_logits_dev [n_seq, V] f32: logits that choose each sequence's first token.
 * slots_host [n_seq]; out_tokens_dev [n_seq, n_new] i32; stats_host (may be NULL)
 * receives {rounds, drafted, accepted} summed over sequences. */
int pulsar_engine_generate_greedy(pulsar_engine* eng, int32_t n_seq, const int32_t* slots_host,
                                  const float* first_logits_dev, int32_t n_new, int32_t gamma,
                                  int32_t* out_tokens_dev, int64_t* stats_host, void* stream);

/* Sampled self-speculative decoding (no reference counterpart: the reference samples with
 * torch.multinomial one token at a time, src/infer.py:594-609, whose warping - temperature,
 * then top-p over the sorted softmax - is kept). gamma >= 1 drafts from the pulse-1 exit,
 * each drawn from its warped distribution q; one batched verify gives p; draft d_j is
 * accepted iff u1 <= min(1, p_{j-1}(d_j) / q_{j-1}(d_j)); the first rejection draws the next
 * token from norm(max(0, p - q)), full acceptance draws it from p_gamma. Every uniform comes
 * from Philox4x32-10 with counter (seq_ids_host[i], round, slot, 0) and key (seed lo, seed hi),
 * u_k = (x_k >> 8) * 2^-24; the first token uses round 0xFFFFFFFF. Draws are inverse-CDF in
 * vocabulary order. temperature > 0, 0 < top_p <= 1, vocab_size <= 49152; a temperature of at
 * most 1e-4 decodes greedily (pulsar_engine_generate_greedy), as the reference's sampler does
 * (src/infer.py:591, 669). Top-p keeps every token whose warped weight is tied with the cutoff
 * token's (the reference sorts, so among exactly tied weights it keeps those the sort puts
 * first). Other arguments as in pulsar_engine_generate_greedy. */
int pulsar_engine_generate_sampled(pulsar_engine* eng, int32_t n_seq, const int32_t* slots_host,
                                   const int32_t* seq_ids_host, const float* first_logits_dev, int32_t n_new,
                                   int32_t gamma, float temperature, float top_p, uint64_t seed,
                                   int32_t* out_tokens_dev, int64_t* stats_host, void* stream);

/* Adaptive early exit (src/infer.py:211-232 set_early_exit_threshold / get_early_exit_stats,
 * the exit rule of decode_step :536-546). enabled != 0: the sequential greedy loop
 * (pulsar_engine_generate_greedy with gamma == 0) ends a token's pulses after pulse k < 2
 * when the softmax of that pulse's (softcapped) logits has max-probability >= threshold;
 * the token is that pulse's argmax and the cached K/V of the position stay the exiting
 * pulse's. The decision runs on the device per sequence; a persistent pulse pass whose rows
 * have all exited returns at once. Speculative rounds (gamma >= 1) run every pulse as
 * before. Each call resets the exit tallies (as the reference's setter does); call it
 * between generate calls, not while one runs on another stream. */
int pulsar_engine_set_early_exit(pulsar_engine* eng, int32_t enabled, float threshold);

/* Repacked weight arena (the checkpoint repack of the engine's load path; the reference
 * reloads and re-merges its .pt checkpoint, src/infer.py:785-817). After finalize the bf16
 * arena - tok_emb (also the LM head), per layer wqkv, wo, shared gate_up / down, routed
 * gate_up / down in the engine's transposed layouts - can be read tensor by tensor; a new
 * engine takes them back with pulsar_engine_arena_write before finalize, in place of the fp32
 * tok_emb / lm_head / wqkv / wo / shared / routed state_dict tensors (the other, small fp32
 * tensors are still uploaded with pulsar_engine_set_tensor). Names: "arena.tok_emb",
 * "arena.<layer>.{wqkv,wo,shared_gate_up,shared_down,routed_gate_up_t,routed_down_t}".
 * arena_info's name pointer stays valid for the engine's lifetime. host buffers hold bf16
 * bit patterns (2 bytes per element). */
int pulsar_engine_arena_count(pulsar_engine* eng, int32_t* count);
int pulsar_engine_arena_info(pulsar_engine* eng, int32_t index, const char** name, int64_t* numel);
int pulsar_engine_arena_read(pulsar_engine* eng, const char* name, void* host_dst, int64_t numel);
int pulsar_engine_arena_write(pulsar_engine* eng, const char* name, const void* host_src, int64_t numel);

/* Repetition penalty of every generate loop (src/infer.py:582-589 and 658-667, the
 * reference's default 1.15 in stream_generate / self_speculative_stream_generate / generate):
 * before each token is chosen, logits of ids already seen are divided by the penalty when
 * positive and multiplied by it otherwise. The seen set of a slot is the prompt of its last
 * pulsar_engine_prefill plus every token that generate calls emitted for it since (a bitmap on
 * the device). In a speculative round the logits that choose the token at block position k
 * (draft or verify) also count the round's drafts before k as seen, so greedy speculative
 * decoding with the penalty emits the penalised sequential stream; sampled calls warp the
 * penalised logits of both the draft and the verify distributions. penalty > 0; 1 turns it
 * off; vocab sizes up to 393,216. */
int pulsar_engine_set_repetition_penalty(pulsar_engine* eng, float penalty);

/* counts_host[3]: tokens that exited after pulse 1, 2 and 3 (the reference's
 * early_exit_counts) since the last pulsar_engine_set_early_exit or create. Waits for the
 * device. */
int pulsar_engine_early_exit_counts(pulsar_engine* eng, int64_t* counts_host);

/* Engine options. "megakernel" (0/1, default 1 when the GPU can co-schedule one CTA per
 * SM): run each pulse pass of <= 5 rows as one persistent kernel instead of per-op
 * kernels. Read-only: "megakernel_grid" (CTAs of the persistent kernel), "loop_adapter"
 * (1 when some loop-adapter lora_B is non-zero; every path, the persistent kernel included,
 * applies it exactly in fp32), "wait_ns" (bound of every wait inside the persistent kernel,
 * 1e5 .. 2e9 ns, default 2e9), "stall_cta" (test hook, default -1: CTA c >= 0 of every persistent
 * launch waits at its first grid barrier for a count the grid never reaches, so the bounded wait
 * runs out and the call reports PULSAR_ERR_CUDA; nothing faults or hangs),
 * "wide" (0/1): run every pulse pass through the many-row GEMM path; read-only "wide_rows"
 * (row capacity of a pass). "kernel_launches" (kernels started by generate_* and pulse since
 * create, each kernel
 * node of a replayed CUDA graph counted per replay), "mega_launches" (the persistent pulse
 * kernels among them), "routed_experts" (distinct routed experts whose weights the persistent
 * kernel streamed, summed over layers and launches; waits for the device). "time_pulses" (0/1):
 * record CUDA events on the caller's stream
 * around every pulse pass launched outside stream capture; "last_pulse_ns" (read-only,
 * waits for the last such pass) is the device time between those events. */
/* "merged_adapter" (0/1, needs a finalized engine): with a live loop adapter (non-zero
 * lora_B), build per-pulse bf16 merged wqkv / wo (src/model.py:716-727 with a bf16 base:
 * bf16 A, bf16(bf16 B * bf16(loop_M[p] * alpha / q)), fp32 product sum in order plus the
 * base, one rounding) and run every pass on them, the persistent kernel included; 0 returns
 * to the exact fp32 adapter correction. Without a live adapter it stays 0. */
/* "tc_gemm" (0/1, default 1): the GEMMs of prefill and the many-row path on the tensor cores
 * (activations split into bf16 hi + lo); 0 selects the fp32 SIMT GEMM. "tma_gemm" (0/1, default
 * 1): the TMA-fed warp-specialised tensor-core GEMM where a tensor map describes the operands;
 * 0 the cp.async-fed one (bit-identical results). "tc_attn" (0/1, default 1): prefill attention
 * on the tensor cores; 0 the fp32 SIMT kernel. */
/* "tc_dec_attn" (0/1, default 1): the decode attention of the per-op and many-row passes on
 * the tensor cores (128-key chunks fed by tensor-map loads, Q and P split into bf16 hi + lo)
 * for a bf16 cache; 0 selects the SIMT kernel. Reads back 1 only when the tensor-core kernel
 * is in use (an fp32 cache always takes the SIMT kernel). */
int pulsar_engine_set_option(pulsar_engine* eng, const char* name, int64_t value);
int pulsar_engine_get_option(pulsar_engine* eng, const char* name, int64_t* value);

/* Phase tracing of the persistent pulse kernel (option "trace" = 1): every launch writes,
 * per CTA, 256 %globaltimer stamps in ns (entry 0: start; 1 + 16*l + j: point j of layer l,
 * j = 0 norm done, 1 QKV tiles, 2 gate, 3 barrier A left, 4 attention items, 5 barrier B left,
 * 6 partials merged, 7 barrier B2 left, 8 Wo tiles and router partials, 9 barrier C left,
 * 10 router logits, 11 up tiles, 12 SwiGLU epilogue, 13 barrier D left, 14 activations
 * loaded, 15 barrier E left; 130 + 8*l + k: steps of the CTA's first attention item (k = 0
 * start, 1 cached keys loaded, 2 queries and new keys, 3 scores, 4 P.V, 5 done); 194 + l:
 * the producer saw layer l's router; 202 LM head start, 203 LM tiles done, 204 argmax
 * ticket, 205 the producer issued its last LM tile; 254: end).
 * host_out must hold megakernel_grid * 256 entries. */
int pulsar_engine_read_trace(pulsar_engine* eng, uint64_t* host_out, int64_t n);

#ifdef __cplusplus
}
#endif

#endif /* PULSAR_B200_H */
