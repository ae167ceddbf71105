/*
 * spec_b200.h -- C ABI of the B200 verify-step backend.
 *
 * A drop-in replacement, for the target-model verify step, of the decoders
 * behind abyo-speculate's `Decoder` / `TreeDecoder` traits
 * (crates/speculate/src/model/mod.rs:39-108 and :118-236) as implemented by
 * `LlamaQuantDecoder` (crates/speculate/src/model/quantized_llama.rs),
 * `Qwen2QuantDecoder` (crates/speculate/src/model/quantized_qwen2.rs) and the
 * BF16 `LlamaDecoder` (crates/speculate/src/model/llama.rs).  Every tensor op
 * runs in this library's own sm_100a CUDA kernels.
 *
 * Conventions
 *  - Plain pointers and sizes only.  The caller owns every host buffer; the
 *    library owns all device memory.  "Rows" of logits are `vocab_size` f32.
 *  - Every function returns a status (SPEC_OK = 0).  On error the decoder
 *    state (history, KV length, cached logits) is unchanged, matching the
 *    trait contract at crates/speculate/src/model/mod.rs:35-38.  No function
 *    aborts or throws across the ABI.  `spec_last_error` gives the message.
 *  - A handle is used by one thread at a time (the trait methods take
 *    `&mut self`; the engine holds `Box<dyn TreeDecoder + Send>`,
 *    crates/speculate/src/engine.rs:97).
 */
#ifndef SPEC_B200_H
#define SPEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Mapping onto crates/speculate/src/error.rs:10-51:
 *   SPEC_ERR_INVALID        -> Error::Sampling (bad argument / protocol misuse)
 *   SPEC_ERR_CACHE_ROLLBACK -> Error::CacheRollback
 *   SPEC_ERR_UNSUPPORTED    -> Error::UnsupportedMethod
 *   SPEC_ERR_IO             -> Error::Io (GGUF open / parse)
 *   SPEC_ERR_CUDA, _OOM, _TIMEOUT -> Error::Other / Error::Candle           */
#define SPEC_OK 0
#define SPEC_ERR_INVALID 1
#define SPEC_ERR_CACHE_ROLLBACK 2
#define SPEC_ERR_UNSUPPORTED 3
#define SPEC_ERR_IO 4
#define SPEC_ERR_CUDA 5
#define SPEC_ERR_OOM 6
#define SPEC_ERR_TIMEOUT 7

/* Largest number of rows (k+1 verify rows, tree nodes, observe chunk) one
 * forward processes; longer observes are chunked internally. */
#define SPEC_MAX_ROWS 64

typedef struct spec_model spec_model;

typedef struct spec_load_opts {
  int device;     /* CUDA device ordinal */
  int max_ctx;    /* KV capacity in tokens; 0 = min(GGUF context_length, 4096) */
  int use_graphs; /* 1 = replay one CUDA graph per row count (default), 0 = eager */
  int tp_rank;    /* tensor-parallel rank of this handle (0 when tp_size <= 1) */
  int tp_size;    /* tensor-parallel ranks (0 or 1 = a whole model on one GPU); see spec_tp_* */
  int reserved[3];
} spec_load_opts;

/* Shape of a seeded synthetic model (weights generated on the device). */
typedef struct spec_model_desc {
  int arch;       /* 0 = llama, 1 = qwen2 */
  int n_layers, hidden, n_heads, n_kv_heads, ffn, vocab;
  float rope_theta;
  float eps;
  int quant_mix;  /* 0 = Q4_K_M, 1 = Q5_K, 2 = Q8_0, 3 = BF16 */
  int rope_half;  /* llama only: 1 = rotate-half RoPE (BF16 checkpoints), 0 = interleaved */
  /* Layers from damp_from_layer on (0 = none) draw their attn_output and
   * ffn_down weights with sigma 0.02 * damp_e4 / 10000: their updates to the
   * residual are small, so a model with the first damp_from_layer layers and
   * the same seed (which shares the embedding, the first layers, the final
   * norm and the head) predicts like this one -- a draft with realistic
   * acceptance for random-weight benchmarks.  Byte counts do not change. */
  int damp_from_layer;
  int damp_e4;
  int reserved[4];
} spec_model_desc;

/* ---- lifetime -------------------------------------------------------------
 * Replaces LlamaQuantDecoder::from_gguf (quantized_llama.rs:57-97) and
 * Qwen2QuantDecoder::from_gguf (quantized_qwen2.rs) -> ModelWeights::from_gguf
 * (quantized_llama_local.rs:217-308, quantized_qwen2_local.rs:210-300).       */
int spec_load_gguf(const char* path, const spec_load_opts* opts, spec_model** out);
/* Synthetic model: seeded N(0, 0.02) weights quantized on the device. */
int spec_create_synthetic(const spec_model_desc* desc, uint64_t seed, const spec_load_opts* opts,
                          spec_model** out);
/* The device generator behind spec_create_synthetic, one tensor at a time,
 * so a test or a CPU checker can rebuild the exact weights a synthetic model
 * (and the benchmark) runs on.  spec_create_synthetic numbers its tensors
 * 1, 2, ... in this order and seeds tensor i with
 * spec_synthetic_seed(model_seed, i):
 *   output_norm (1 + N(0, 0.02)), token_embd, output (N(0, 0.02) matrices,
 *   [rows][K] GGUF blocks), then per layer: attn_q, attn_k, attn_v,
 *   attn_output, ffn_gate, ffn_up, ffn_down (N(0, 0.02); attn_output and
 *   ffn_down of damped layers N(0, 0.02 * damp_e4 / 10000)), attn_norm,
 *   ffn_norm (1 + N(0, 0.02)), and for qwen2 one q|k|v bias vector
 *   (N(0, 0.02)).  Models with the same seed and shape but fewer layers
 *   therefore share the embedding, head, final norm and first layers.
 * Types follow the quant mix: Q4_K_M = Q4_K, with Q6_K for attn_v and
 * ffn_down on even layers and for output; Q8_0 wherever K % 256 != 0.
 * No counterpart in the reference (its weights come from checkpoints). */
uint64_t spec_synthetic_seed(uint64_t model_seed, uint64_t index);
/* Raw GGUF blocks of one N(0, sigma) tensor of `rows` x `k_cols`, generated on
 * `device` and copied to host_out (out_bytes >= rows * k_cols / block elements
 * * block bytes). */
int spec_synthetic_tensor(int device, int ggml_type, int rows, int k_cols, uint64_t seed, float sigma,
                          void* host_out, int64_t out_bytes);
/* base + N(0, sigma) f32 vector of n elements (norm weights, biases). */
int spec_synthetic_vector(int device, int n, uint64_t seed, float base, float sigma, float* host_out);
void spec_free(spec_model* m);

/* ---- tensor parallelism (one process per GPU) ----------------------------
 * No counterpart in the reference (candle runs the model on one device).  A
 * handle loaded with tp_size > 1 holds rank tp_rank's shard: its q/kv heads
 * and FFN slice (column-parallel q/k/v and gate/up, row-parallel o and down,
 * KV cache of its heads; embedding and norms whole) and its 128-row-aligned
 * slice of the LM head (vocabulary-parallel: each rank computes its rows of
 * the logits and stores them into every rank's logits buffer, so every rank
 * returns the full rows).  The sums of
 * the row-parallel projections are exchanged inside the forward kernel over
 * NVLink peer memory.  Before the first forward every rank exports its
 * receive buffer (spec_tp_handle: writes an opaque handle, returns its byte
 * count or a negated status) and connects to all ranks' handles, given in
 * rank order (spec_tp_connect).  Every rank must then make the same calls
 * with the same arguments; results are identical on all ranks. */
int spec_tp_handle(spec_model* m, void* out, int cap);
int spec_tp_connect(spec_model* m, const void* handles, int n);
int spec_tp_size(const spec_model* m);
/* Message of the last error on `m`; with m == NULL, of the last failed
 * load on the calling thread. */
const char* spec_last_error(const spec_model* m);

/* ---- shape / state queries -------------------------------------------------
 * Decoder::vocab_size, ::history, ::history_len (model/mod.rs:41-50);
 * TreeDecoder::num_hidden_layers (mod.rs:177-182).                           */
int spec_vocab_size(const spec_model* m);
int spec_hidden_size(const spec_model* m);
int spec_num_layers(const spec_model* m);
int spec_history_len(const spec_model* m);
/* Copies min(cap, history_len) tokens; returns the full history length. */
int spec_history(const spec_model* m, uint32_t* out, int cap);
/* Current KV length (the reference decoder's `cache_len`).  A token that
 * spec_observe left pending (see below) counts. */
int spec_kv_len(const spec_model* m);
int spec_max_ctx(const spec_model* m);

/* ---- Decoder (model/mod.rs:39-108) ---------------------------------------- */
/* Decoder::reset (mod.rs:52-53; quantized_llama.rs:512-517). */
int spec_reset(spec_model* m);
/* Decoder::observe (mod.rs:55-56; quantized_llama.rs:519-526).  Lazy: the KV
 * rows of all but the last new token are computed now; the last one is
 * computed inside the next call that needs it (next_logits, batched_logits,
 * tree or verify forwards recompute the last committed token anyway), so the
 * observe after a vanilla SD round costs no forward of its own.  Observable
 * results (logits, history, KV length, errors) are those of an eager observe. */
int spec_observe(spec_model* m, const uint32_t* ids, int n);
/* Decoder::next_logits (mod.rs:58-60; quantized_llama.rs:528-551); out: V f32. */
int spec_next_logits(spec_model* m, float* out);
/* Decoder::batched_logits (mod.rs:62-74; quantized_llama.rs:553-583);
 * out: (k+1) x V f32.  Afterwards history += drafts. */
int spec_batched_logits(spec_model* m, const uint32_t* drafts, int k, float* out);
/* Decoder::rollback_to (mod.rs:76-80; quantized_llama.rs:585-599). */
int spec_rollback_to(spec_model* m, int len);

/* ---- TreeDecoder (model/mod.rs:118-236) ------------------------------------
 * A draft tree is (tokens[n], parents[n]) in BFS order with parents[0]
 * ignored and parents[i] < i (crates/speculate/src/tree.rs:38-74).          */
/* TreeDecoder::tree_logits (mod.rs:135-144; quantized_llama.rs:262-325);
 * out: n x V.  History and KV are restored.  A tree of more than
 * SPEC_MAX_ROWS nodes runs as several forwards over ancestor-closed chunks
 * (each node with all its ancestors, at most SPEC_MAX_ROWS rows); only a node
 * more than SPEC_MAX_ROWS - 1 levels deep is refused (SPEC_ERR_UNSUPPORTED).
 * spec_tree_logits_keep_kv, spec_verify_tree_greedy and spec_commit_tree_path
 * take such trees too: the KV window then holds the last chunk's rows
 * (spec_kv_len = prefix + that chunk's size), and the commit, whose accepted
 * nodes must then form a path from the root, re-runs the path's chunk when
 * the window holds another.  spec_verify_tree_typical, spec_medusa_round
 * and spec_eagle_round do the same. */
int spec_tree_logits(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float* out);
/* TreeDecoder::tree_logits_keep_kv (mod.rs:196-210; quantized_llama.rs:341-394);
 * logits_out: n x V (may be NULL), hidden_out: n x hidden (may be NULL).
 * KV is left holding the prefix plus all n tree nodes. */
int spec_tree_logits_keep_kv(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                             float* logits_out, float* hidden_out);
/* TreeDecoder::commit_tree_path (mod.rs:223-235; quantized_llama.rs:409-440).
 * accepted: node indices root-first (accepted[0] == 0). */
int spec_commit_tree_path(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                          const int32_t* accepted, int n_acc);
/* TreeDecoder::last_hidden_state (mod.rs:127-133; quantized_llama.rs:193-212). */
int spec_last_hidden_state(spec_model* m, float* out);
/* TreeDecoder::observe_returning_last_hidden (mod.rs:212-221; quantized_llama.rs:174-191). */
int spec_observe_returning_last_hidden(spec_model* m, const uint32_t* ids, int n, float* hidden_out);
/* TreeDecoder::apply_lm_head (mod.rs:146-156; quantized_llama.rs:112-121):
 * rows x hidden f32 -> rows x V f32. */
int spec_apply_lm_head(spec_model* m, const float* hidden, int rows, float* out);
/* TreeDecoder::apply_lm_head followed by methods::medusa::top_k_indices
 * (medusa.rs:477-487), as the EAGLE draft loop uses them (eagle.rs:549-566),
 * with the top-k on the device: ids_out[rows][k] (and, when non-NULL,
 * vals_out[rows][k]) in descending logit order, ties by ascending index.
 * 1 <= k <= 64.  Only rows x k ids (and values) cross to the host instead of
 * rows x V logits.  NaN logits rank below every number. */
int spec_apply_lm_head_topk(spec_model* m, const float* hidden, int rows, int k, int32_t* ids_out, float* vals_out);
/* TreeDecoder::embed_tokens (mod.rs:184-194; quantized_llama_local.rs:328-330). */
int spec_embed_tokens(spec_model* m, const uint32_t* ids, int n, float* out);
/* TreeDecoder::last_hidden_states_multi (mod.rs:158-175; quantized_llama.rs:221-249):
 * final_out: hidden f32; layer_outs: n_sel x hidden f32 (residual after layer). */
int spec_last_hidden_states_multi(spec_model* m, const int32_t* layers, int n_sel, float* final_out,
                                  float* layer_outs);

/* ---- EAGLE draft on the device (methods/eagle.rs) ----------------------------
 * The EAGLE draft block (eagle.rs:390-427): concat(target hidden, token
 * embedding) -> fc -> one Llama block without input norm (RoPE rotate-half in
 * the checkpoint's BF16, its own per-round KV cache) -> post-attention
 * RMSNorm -> SiLU MLP, with shapes equal to a target layer.  Weights are BF16
 * (row-major [out][in] bits), the norm f32; the token embedding is the
 * target's.  rope_theta <= 0 takes the target's. */
typedef struct spec_eagle_weights {
  const uint16_t* fc;    /* [H][2H] */
  const uint16_t* q;     /* [n_heads*hd][H] */
  const uint16_t* k;     /* [n_kv*hd][H] */
  const uint16_t* v;     /* [n_kv*hd][H] */
  const uint16_t* o;     /* [H][n_heads*hd] */
  const uint16_t* gate;  /* [F][H] */
  const uint16_t* up;    /* [F][H] */
  const uint16_t* down;  /* [H][F] */
  const float* post_norm; /* [H] */
  float rope_theta;
} spec_eagle_weights;
int spec_eagle_attach(spec_model* m, const spec_eagle_weights* w);
/* Seeded N(0, 0.02) BF16 weights made on the device (benchmarks). */
int spec_eagle_attach_synthetic(spec_model* m, uint64_t seed);
/* One round's draft loop (eagle.rs:531-575) on the device: depth steps of the
 * draft block, each followed by the target's LM head, a device top-k
 * (medusa.rs:477-487 order) and log-softmax; the next step takes the top-1
 * token and the draft's hidden row without leaving the device.  hidden: the
 * target's last hidden row [H]; root: the last committed token; position: the
 * target's history length.  Writes ids_out[depth][k] and (when non-NULL)
 * logprobs_out[depth][k] = logit - logsumexp(row).  depth <= 64. */
int spec_eagle_draft(spec_model* m, const float* hidden, uint32_t root, int position, int depth, int k,
                     int32_t* ids_out, float* logprobs_out);
/* The round's draft tree (methods/eagle.rs:584-593, host code): the
 * Cartesian product of the depth steps' top-k (medusa.rs:172-189, BFS
 * layers), and when max_nodes > 0 and the product is larger, its pruning by
 * path log-prob (eagle.rs:763-843: f32 sums deepest step first, stable
 * descending order, the best max_nodes - 1 plus their ancestors, BFS order).
 * ids / logprobs: [depth][k] as spec_eagle_draft writes them.  Writes the
 * tree as tokens / parents (parents[0] = 0) and its size; a tree larger than
 * cap, or a product above 2^26 nodes, returns SPEC_ERR_UNSUPPORTED. */
int spec_eagle_build_tree(uint32_t root, const int32_t* ids, const float* logprobs, int depth, int k, int max_nodes,
                          uint32_t* tokens_out, int32_t* parents_out, int cap, int* n_out);
/* One EAGLE-2 round at temperature 0 as one native call (run_eagle's loop
 * body, methods/eagle.rs:531-731), on a target with an attached EAGLE head:
 *   the draft loop from `hidden` (the target's last hidden row [H]) with the
 *   last committed token as root; the tree of spec_eagle_build_tree (up to
 *   16384 nodes; over SPEC_MAX_ROWS it runs as ancestor-closed chunks, as
 *   spec_tree_logits does, and the bonus is always observed); the tree
 *   forward keeping KV and the greedy walk of
 *   spec_verify_tree_greedy; committed = the accepted path's tokens + the
 *   bonus, cut after the first token of eos_ids;
 *   the KV commit (:680-727): an EOS on the path keeps the path up to it;
 *   otherwise, unless strict_root, a child of the deepest accepted node
 *   holding the bonus joins the commit and its tree hidden row is the next
 *   hidden; else the path is committed and the bonus observed.
 * strict_root only disables that shortcut: the backend's tree row 0 equals
 * next_logits bit for bit, so the reference's strict root logits change
 * nothing else.  Writes commits_out (room for depth + 1), *n_out,
 * hidden_out [H] (the next round's hidden; not written when an EOS on the
 * path stops the round) and *stop (an EOS was committed). */
int spec_eagle_round(spec_model* m, const float* hidden, int depth, int top_k, int max_tree_nodes, int strict_root,
                     const uint32_t* eos_ids, int n_eos, uint32_t* commits_out, int* n_out, float* hidden_out,
                     int* stop);

/* ---- Medusa draft heads on the device (methods/medusa.rs) -------------------
 * Each head (MedusaHeadModule, medusa.rs:509-584) maps the target's last
 * hidden row through residual_layers blocks x' = x + SiLU(W x + b)
 * (W [H][H], b [H]) and an output projection [V][H] without bias; weights are
 * BF16 (row-major [out][in] bits), biases f32.  1 <= n_heads <= 8,
 * 0 <= residual_layers <= 4.  res_w / res_b list [head][layer]. */
typedef struct spec_medusa_weights {
  int n_heads;
  int residual_layers;
  const uint16_t* const* res_w;  /* [n_heads * residual_layers] -> [H][H] */
  const float* const* res_b;     /* [n_heads * residual_layers] -> [H] */
  const uint16_t* const* out_w;  /* [n_heads] -> [V][H] */
} spec_medusa_weights;
int spec_medusa_attach(spec_model* m, const spec_medusa_weights* w);
/* Seeded N(0, 0.02) BF16 weights and biases made on the device (benchmarks). */
int spec_medusa_attach_synthetic(spec_model* m, int n_heads, int residual_layers, uint64_t seed);
/* MedusaHeadsCandle::top_k_per_head (medusa.rs:713-734): every head applied to
 * hidden [H], then top_k_indices (medusa.rs:477-487) over its logits on the
 * device.  Writes ids_out[n_heads][k] (descending logit, ties by ascending
 * index) and, when non-NULL, logprobs_out[n_heads][k] = logit - logsumexp.
 * 1 <= k <= 64. */
int spec_medusa_topk(spec_model* m, const float* hidden, int k, int32_t* ids_out, float* logprobs_out);
/* Number of attached Medusa heads (0 when none). */
int spec_medusa_num_heads(const spec_model* m);
/* One Medusa round, the body of run_medusa_real's loop
 * (crates/speculate/src/methods/medusa.rs:761-810), in one call: the heads'
 * top_k from `hidden` (the target's last hidden row, host, hidden_size
 * floats), the draft tree of `topology` (0 = Greedy: each head's top-1 as a
 * chain, :167-170; 1 = CartesianProduct: BFS layers, every candidate of head
 * d under every node of layer d, :172-189), the tree forward keeping KV, the
 * walk with `acceptance` (0 = Greedy, as spec_verify_tree_greedy; 1 =
 * Typical {epsilon, delta}, as spec_verify_tree_typical), the commit of the
 * accepted path and, while fewer than `budget` (max_new_tokens - generated)
 * tokens are committed, the argmax bonus of the deepest accepted node.
 * commits_out (room for n_heads + 1) receives the committed tokens, *n_out
 * their count, hidden_out (hidden_size floats) the hidden row of the last
 * committed token: the next round's `hidden`.  History and KV afterwards are
 * those of the reference's observe(committed).  Trees over SPEC_MAX_ROWS
 * nodes run as ancestor-closed chunks (spec_tree_logits); one over 16384
 * nodes returns SPEC_ERR_UNSUPPORTED with the state unchanged. */
int spec_medusa_round(spec_model* m, const float* hidden, int top_k, int topology, int acceptance, float epsilon,
                      float delta, int budget, uint32_t* commits_out, int* n_out, float* hidden_out);

/* ---- device-side acceptance ------------------------------------------------
 * Greedy (temperature 0) vanilla verify: one batched forward of [last]+drafts
 * (same protocol and state change as spec_batched_logits), then the argmax of
 * every row on the device (first-max tie break, crates/speculate/src/
 * sampling/tokens.rs:25-36) and the accept walk of methods/vanilla.rs:312-343
 * at temperature 0.  Writes n_accepted (0..k) and the token that follows
 * them (the argmax of row n_accepted).  Row argmaxes go to argmax_out[k+1]
 * when it is non-NULL.  Only (k+1) ints cross to the host. */
int spec_verify_greedy(spec_model* m, const uint32_t* drafts, int k, int* n_accepted, uint32_t* next_token,
                       int32_t* argmax_out);
/* One greedy vanilla SD round over a target and a draft handle
 * (methods/vanilla.rs:285-369 at temperature 0): k draft steps (device
 * argmax + lazy observe), spec_verify_greedy on the target, then both roll
 * back to the accepted prefix and observe the next token.  Writes the
 * committed tokens (accepted drafts, then the next token) to commits_out
 * (room for k+1) and their count to *n_out.  The histories must be equal on
 * entry; they are equal again on return. */
int spec_sd_greedy_round(spec_model* target, spec_model* draft, int k, uint32_t* commits_out, int* n_out);
/* Greedy tree acceptance of methods/eagle.rs:618-661 over a tree forward
 * (spec_tree_logits_keep_kv semantics, KV kept): best_path receives the
 * accepted node indices root-first (capacity n), *path_len its length, and
 * *bonus the argmax of the deepest accepted node. */
int spec_verify_tree_greedy(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                            int32_t* best_path, int* path_len, uint32_t* bonus);
/* Medusa typical acceptance (crates/speculate/src/methods/medusa.rs:290-326
 * with Acceptance::Typical { epsilon, delta }, accept_one at :424-445) over
 * the same tree forward (KV kept): node i passes iff, under its parent's
 * row, p(token_i) >= max(epsilon, delta * exp(-H(p))), with the softmax and
 * the entropy in the reference's f32 operations and sequential order (max,
 * exp(l - max), sequential sum, division; sequential sum of (-p) * ln(p) over
 * p > 0); a row with non-positive or non-finite mass rejects every child.
 * Walk, outputs and state change as spec_verify_tree_greedy; the bonus is the
 * argmax of the deepest accepted node (medusa.rs:311-316, :451-470). */
int spec_verify_tree_typical(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float epsilon,
                             float delta, int32_t* best_path, int* path_len, uint32_t* bonus);
/* Rejection-sampling vanilla round (methods/vanilla.rs:172-210 steps 3-4) on
 * the device: one batched forward of [last]+drafts (same protocol and state
 * change as spec_batched_logits), then, with the reference's float32
 * operations in its order (sampling/tokens.rs:14-55 and :99-120,
 * vanilla.rs:59-106):
 *   for i < k: p = softmax_t(target row i); accept drafts[i] iff
 *     q_i[x] <= 0 or u <= min(p[x] / q_i[x], 1) with the next uniform;
 *     on the first rejection, commit a sample (next uniform) of
 *     norm(max(p - q_i, 0)) and stop;
 *   if all k were accepted and fewer than `budget` tokens are committed,
 *     commit a bonus sample (next uniform) of softmax_t(target row k).
 * A commit that reaches `budget` (the round's max_new - generated) ends the
 * round, as the reference's loop does.  draft_probs: k x V f32 (the draft
 * distributions q_i, host); uniforms: the round's gen::<f32>() draws in the
 * reference order (at most k + 1 are used).  Writes the committed tokens to
 * commits (capacity k + 1), their count, and the number of uniforms used.
 * temperature 0 is the one-hot argmax distribution.  Errors of the
 * reference's sampling (invalid temperature, non-positive softmax or adjusted
 * mass, too few uniforms) return SPEC_ERR_INVALID with the state unchanged. */
int spec_verify_rejection(spec_model* m, const uint32_t* drafts, int k, const float* draft_probs,
                          float temperature, const float* uniforms, int n_uniforms, int budget, uint32_t* commits,
                          int* n_commits, int* n_uniforms_used);

/* ---- seeded sampling stream and the sampled SD round --------------------- */
/* The reference's sampling RNG, StdRng::seed_from_u64(seed)
 * (crates/speculate/src/engine.rs:320-326; rand 0.8.6 StdRng = ChaCha12 of
 * rand_chacha 0.3.1, seeded by rand_core 0.6's PCG32 fill), drawn with
 * gen::<f32>() = (next_u32 >> 8) * 2^-24 (sampling/tokens.rs:99-120).  Host
 * state only: usable without a GPU. */
typedef struct spec_rng spec_rng;
int spec_rng_create(uint64_t seed, spec_rng** out);
void spec_rng_free(spec_rng* r);
/* The next n gen::<f32>() draws (consumed). */
int spec_rng_next_f32(spec_rng* r, float* out, int n);
/* One vanilla SD round at temperature >= 0 as one native call
 * (methods/vanilla.rs:285-369 with the engine's seeded stream):
 *   k' = min(k, budget) draft steps, each a forward of the draft's pending
 *     token, softmax_t of its row and a sample with the next draw
 *     (sampling/tokens.rs:14-55, 99-120), observed lazily; the draft's
 *     probability rows stay on the device;
 *   spec_verify_rejection on the target with those rows and the next draws
 *     (one per verified position, then one for the resample or the bonus);
 *   the stream advances by the draws used; both decoders roll back to
 *     pre + min(n_commits, k') and observe the commits past it
 *     (vanilla.rs:352-362: a resampled token is emitted, not observed).
 * Writes the committed tokens (room for k+1), their count and the number of
 * drafts accepted.  The histories must be equal on entry. */
int spec_sd_sampled_round(spec_model* target, spec_model* draft, int k, float temperature, spec_rng* rng, int budget,
                          uint32_t* commits_out, int* n_out, int* n_accepted);

/* ---- diagnostics -------------------------------------------------------- */
/* Device time (ms, CUDA events) of the most recent forward. */
float spec_last_forward_ms(const spec_model* m);
/* The CUDA stream (cudaStream_t) every forward of `m` runs on, for callers
 * that bracket calls with their own CUDA events. */
void* spec_cuda_stream(const spec_model* m);
/* One eager verify forward of [last] + drafts (the spec_batched_logits
 * protocol, but the decoder's history / KV length are left unchanged and the
 * cached next logits are dropped), with a CUDA event after every kernel.
 * Writes per-launch device ms, kind (0 embed, 2 attention split+combine,
 * 8 one persistent multi-op GEMV launch: a layer's o-proj, gate/up and down
 * plus the next layer's qkv, or the LM head) and algorithmic bytes (packed
 * weights, or KV bytes for attention); returns the number of launches, or a
 * negated status on error. */
int spec_profile_forward(spec_model* m, const uint32_t* drafts, int k, float* ms_out, int* kind_out,
                         int64_t* bytes_out, int cap);
/* Number of kernel launches one forward of `rows` rows performs. */
int spec_kernels_per_forward(const spec_model* m, int rows);
/* Total weight bytes streamed by one forward (packed weights, all layers + head). */
int64_t spec_weight_bytes(const spec_model* m);

/* ---- standalone dequant-matmul (QMatMul::forward, candle 0.8.4) -----------
 * y[M][N] = x[M][K] . W^T on device buffers, for the microbench and tests.
 * W is uploaded once from raw GGUF blocks (row-major [N][K/blk]).           */
typedef struct spec_qweight spec_qweight;
int spec_qweight_upload(int ggml_type, const void* gguf_blocks, int n_rows, int k_cols, int device,
                        spec_qweight** out);
void spec_qweight_free(spec_qweight* w);
/* x_dev: M x K f32 (device), y_dev: M x N f32 (device); stream may be NULL
 * (the weight's own stream, synchronised on return).  The weight's device is
 * current during the call and the caller's current device is restored.  With
 * stream == NULL a device wait that gave up inside the kernel (y incomplete)
 * returns SPEC_ERR_TIMEOUT and clears the weight's error word; with a caller
 * stream nothing is synchronised and such a timeout is reported by the next
 * synchronous call on the same weight.  Messages: spec_last_error(NULL). */
int spec_qmatmul(spec_qweight* w, const float* x_dev, int M, float* y_dev, void* stream);
/* Weight bytes of the packed matrix (equal to the GGUF byte count). */
int64_t spec_qweight_bytes(const spec_qweight* w);
/* Average device ms of the dequant kernel over `iters` launches of the last
 * spec_qmatmul shape (CUDA events on the launching stream). */
int spec_qmatmul_time(spec_qweight* w, int M, int iters, int flush_l2, float* avg_ms);

/* ---- no-allocation matmul (no counterpart in the reference) ---------------
 * spec_qmatmul_noalloc: the spec_qmatmul contract (same arguments, result
 * within the same tolerance; it runs the same kernel), but the call
 * allocates no memory.  spec_qmatmul allocates a descriptor slot and pinned
 * staging on its first call; this entry point keeps every piece of per-call
 * scratch (operand fragments and column sums, split-K partials and counters,
 * the op descriptor) in one file-scope device array of
 * SPEC_NOALLOC_SCRATCH_BYTES per device.  It is for callers that cannot
 * allocate:
 *   - a serving runtime that reserves nearly all device memory up front
 *     (weights, KV pages), where a late cudaMalloc fails or forces eviction;
 *   - a latency-critical loop that must not meet the device-wide
 *     synchronisation that cudaFree (and at times cudaMalloc) implies;
 *   - code running inside an allocator or memory-pool callback, where
 *     re-entering the allocator deadlocks.
 * Limits and rules:
 *   - a call needs about 2.4*K*m8 bytes of operand (m8 = M rounded up to
 *     8, 16, 32 or 64) plus, when the weight's work is cut into C > 1
 *     chunks (C <= resident CTAs, 444 on a B200 at M <= 8),
 *     (C + N/128)*512*m8 bytes of partials; a shape needing more than
 *     SPEC_NOALLOC_SCRATCH_BYTES returns SPEC_ERR_INVALID (message via
 *     spec_last_error(NULL)) and launches nothing;
 *   - the first call on a device looks the array up (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream
 *     capture begins;
 *   - every call on a device shares the one array: calls on the same stream
 *     are ordered, but calls that overlap in time (different streams, or
 *     several host threads) race on it and corrupt each other's results;
 *   - each call zeroes the counters it uses (an async memset on `stream`)
 *     and rewrites everything else it reads before reading it;
 *   - stream may be NULL (the weight's own stream, synchronised on return);
 *     each call clears the weight's error word before its launch, so a
 *     synchronous call reports a device wait that gave up in its own launch
 *     as SPEC_ERR_TIMEOUT; with a caller stream such a timeout is not
 *     reported (the next call clears the word first);
 *   - the looked-up address belongs to the device's primary context: calls
 *     must not cross a cudaDeviceReset of that device;
 *   - the caller's current device is restored on return.
 * Error messages are thread-local (spec_last_error(NULL)). */
#define SPEC_NOALLOC_SCRATCH_BYTES (16u << 20)
int spec_qmatmul_noalloc(spec_qweight* w, const float* x_dev, int M, float* y_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPEC_B200_H */
