// Kernel parameter blocks and launchers of the verify-step backend.
//
// Data layout in HBM (one model):
//   * weights: every quantized matrix is repacked at load into "pair tiles"
//     of 32 rows x KT columns laid out in mma-fragment order (see qgemv.cu);
//     the byte count equals the GGUF byte count (same bits per weight).  BF16
//     matrices are repacked per 128-row x 128-column stage into the tensor
//     core's K-major no-swizzle canonical layout (tcgen05 operands).
//   * residual stream h: f32 [M][H].
//   * activation operand of every GEMV: f16 values in m16n8k16 B-fragment
//     order, or bf16 values (BF16 models) in the canonical layout
//     (operand_half_index), plus per-16 / per-32 column sums of those
//     rounded values, stored already multiplied by the tiles' accumulator
//     seeds: xsum16 = -1056 x (sum of 16), xsum32 = -1024 x (sum of 32)
//     (kXSum16Seed / kXSum32Seed), so a tile loads its MMA's C operand.
//   * KV cache: f16 (bf16 for BF16 models) [layer][kv_head][t][head_dim], K and
//     V in separate arenas; rows beyond the live length hold finite stale data.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace specb200 {

// Error bits reported through the per-model device error word.
enum DevError : unsigned {
  DEV_ERR_MBAR_TIMEOUT = 1u << 0,   // an mbarrier wait gave up
  DEV_ERR_BAD_ARGUMENT = 1u << 1,   // a kernel saw an out-of-range index
};

// The error word is err[0]; a wait that gives up also records where, once:
// err[1] = site | op << 8 | cta << 16, err[2] = stage / ring position,
// err[3] = the counter value it last saw.
// (Site 2 was the consumers' per-op dependency wait, which per-group flags
// made unnecessary; the number stays retired.)
// Site 6: the producer's last wait for its own copies to land before exit.
enum WaitSite : unsigned {
  WAIT_CONSUMER_FULL = 1,
  WAIT_PRODUCER_IDLE = 3,
  WAIT_TP_PEERS = 4,
  WAIT_ATTN_DEP = 5,
  WAIT_PRODUCER_DRAIN = 6
};

// GGML type ids (public GGUF specification) of the weight formats handled.
enum WFmt : int { WF_F32 = 0, WF_F16 = 1, WF_Q8_0 = 8, WF_Q4_K = 12, WF_Q5_K = 13, WF_Q6_K = 14, WF_BF16 = 30 };

// Columns per tile and bytes per 16-row tile of each repacked format.
__host__ __device__ constexpr int fmt_kt(int f) { return f == WF_Q8_0 ? 128 : (f == WF_BF16 ? 128 : 256); }
__host__ __device__ constexpr int fmt_tile_bytes(int f) {
  return f == WF_Q4_K ? 2304 : f == WF_Q5_K ? 2816 : f == WF_Q6_K ? 3360 : f == WF_Q8_0 ? 2176 : f == WF_BF16 ? 4096 : 0;
}
__host__ __device__ constexpr int fmt_pair_bytes(int f) { return 2 * fmt_tile_bytes(f); }
__host__ __device__ constexpr int fmt_stages(int f) { return f == WF_Q6_K || f == WF_Q5_K ? 2 : 3; }
__host__ __device__ constexpr int fmt_block_elems(int f) {
  return (f == WF_Q4_K || f == WF_Q5_K || f == WF_Q6_K) ? 256 : f == WF_Q8_0 ? 32 : 1;
}
__host__ __device__ constexpr int fmt_block_bytes(int f) {
  return f == WF_Q4_K ? 144 : f == WF_Q5_K ? 176 : f == WF_Q6_K ? 210 : f == WF_Q8_0 ? 34 : f == WF_F32 ? 4 : 2;
}

constexpr int kGemvWarps = 4;          // warps per CTA
constexpr int kGroupRows = 128;        // rows per CTA (4 warps x 32 rows)
constexpr int kMaxRows = 64;           // max activation rows (M) per forward
constexpr int kSsStride = 64;          // stride of per-group sum-of-squares slots
constexpr int kMaxSsGroups = 64;       // hidden size <= 64 * 128
// Seeds the operand column sums carry (see the layout note at the top):
// Q6_K codes sit at 1024 + 32 + q, Q4_K/Q5_K codes at 1024 + q.
constexpr float kXSum16Seed = -1056.f;
constexpr float kXSum32Seed = -1024.f;
constexpr int kTpSlot = kMaxRows * 128;  // words per (source rank, group) receive slot
constexpr int kTpMaxLayers = 256;        // tp_tag = 2 x layer + set stays below 512
constexpr int kTpMaxRanks = 8;           // tensor-parallel ranks per model
__host__ __device__ inline unsigned tp_flag_of(unsigned epoch, int tag) { return (epoch << 9) | (unsigned)tag; }

// Number of 8-row fragment columns (n-tiles) the kernels use for M rows: the
// GEMV is instantiated for 1, 2, 4 and 8, and every producer of an operand
// must lay it out for the same count.
__host__ __device__ constexpr int nt_for_rows(int M) { return M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8; }

// Position (in 16-bit elements) of operand element (row m, column k) of an
// operand laid out for nt_total n-tiles.  Both layouts spend 256 bytes per
// (16-column k-step, n-tile), k-steps outermost:
//  * f16 operands (consumed by the mma.sync tiles of the quantized formats):
//    m16n8k16 B-fragment order, lane (g = m % 8, t) holding columns 2t, 2t+1,
//    2t+8, 2t+9 of row g in one 8-byte word;
//  * bf16 operands (consumed by the tcgen05 path of BF16 weights): the K-major
//    no-swizzle canonical layout of the tensor core's shared-memory
//    descriptors, two 8x8 core matrices per (k-step, n-tile) (columns 0-7,
//    then 8-15), each 8 rows of 16 bytes.
__host__ __device__ inline size_t operand_half_index(int nt_total, int m, int k, bool bf16) {
  const int s = k >> 4, kk = k & 15, nt = m >> 3, g = m & 7;
  if (bf16) return ((size_t)((s * nt_total + nt) * 2 + (kk >> 3))) * 64 + g * 8 + (kk & 7);
  const int t = (kk & 7) >> 1, slot = kk >> 3, lo = kk & 1;
  return ((size_t)((s * nt_total + nt) * 32 + g * 4 + t)) * 4 + slot * 2 + lo;
}

// Epilogue applied by the CTA that owns the final sum of a 128-row group.
enum Epi : int {
  EPI_STORE = 0,   // out[m*ld + n] = rinv[m]*y + bias[n]
  EPI_QKV = 1,     // bias, RoPE, q -> qbuf, k/v -> cache
  EPI_RESID = 2,   // h += y; per-group sum of squares; next operand fragments
  EPI_SILU = 3,    // silu(gate) * up -> next operand fragments
};

struct WSeg {                // one weight segment (one format)
  const uint8_t* w = nullptr;  // pair tiles
  int fmt = 0;
  int groups = 0;              // 128-row groups in this segment
  int k_tiles = 0;             // K / KT
};

struct QmvParams {
  WSeg seg[2];
  int n_rows = 0;        // total output rows (both segments)
  int K = 0;
  // Work split (stream-K): the op's stages (one k-tile of one 128-row group;
  // segment 0's groups first, each group's k-tiles in order) are cut into
  // `chunks` contiguous runs, chunk i = [i*stages/chunks, (i+1)*stages/chunks).
  // The cut depends on the matrix only, never on M or the grid, so every
  // row's f32 summation order is fixed.
  int stages = 0;
  int chunks = 1;
  int M = 1;
  // activation operand
  const uint32_t* xfrag = nullptr;
  const float* xsum16 = nullptr;
  const float* xsum32 = nullptr;
  // rinv of an RMSNorm folded into this GEMV's input (null = none)
  const float* ss_in = nullptr;
  // The input operand was emitted pre-scaled by the rinv of this table (the
  // previous residual's); the epilogue undoes it (null = not pre-scaled).
  const float* ss_pre = nullptr;
  // EPI_RESID: scale the emitted next operand by the rinv of this table (the
  // residual before this op's update), keeping f16 operands O(1) however large
  // the residual grows (null = no scaling).
  const float* ss_scale = nullptr;
  // Tensor parallelism (EPI_RESID of the row-parallel o / down projections):
  // after this rank's split reduction, the group's sum is stored into every
  // rank's receive slot over NVLink, and the ranks' sums are added in rank
  // order before the residual update, the same way on every rank.  Each
  // 8-byte slot word carries a value (low half) and the flag of its use
  // (high half: tp_flag_of(*tp_epoch, tp_tag)), so a reader needs no fence
  // or counter: a word is ready when its flag is the current one.
  int tp_size = 1, tp_rank = 0;
  int tp_tag = 0;                                    // 2 x layer + set: distinct within one forward
  const unsigned* tp_epoch = nullptr;                // forward counter, identical on every rank
  unsigned long long* const* tp_recv = nullptr;      // [tp_size] device: rank r's receive set
  const unsigned long long* tp_recv_local = nullptr; // this rank's set [src rank][group][kTpSlot]
  // Vocabulary-parallel LM head (EPI_STORE under tensor parallelism): each
  // rank computes its own rows of the logits and stores them into every
  // rank's logits buffer (out_peers[r] = rank r's buffer at this rank's first
  // row), then adds each finished group to every rank's arrival counter
  // (out_counters[r]); tp_logits_wait() holds a rank's stream until all
  // ranks' groups of this forward have arrived.
  // Set only on the head op, whose tp_size stays 1 (tp_size > 1 selects the
  // row-parallel exchange above).
  int out_ranks = 0;                                   // ranks of out_peers / out_counters
  float* const* out_peers = nullptr;                   // [out_ranks] device
  unsigned long long* const* out_counters = nullptr;   // [out_ranks] device
  int ss_groups = 0;
  float ss_inv_dim = 0.f;
  float eps = 0.f;
  // split-K scratch: partial sums, slot (chunk + group) x [128 rows][8*NT]
  // (chunks + groups slots), and one arrival counter per group (zero between ops)
  float* part = nullptr;
  int* counters = nullptr;
  unsigned* err = nullptr;
  // epilogue
  int epi = EPI_STORE;
  float* out = nullptr;
  int ld_out = 0;
  const float* bias = nullptr;
  // EPI_QKV
  int n_q_heads = 0, n_kv_heads = 0, head_dim = 0;
  int rope_interleaved = 0;       // 1: pairs (2i,2i+1) (rope_i); 0: pairs (i, i+d/2)
  const float* rope_cos = nullptr;  // [ctx][head_dim/2]
  const float* rope_sin = nullptr;
  const int* positions = nullptr;   // [M] RoPE positions
  const int* kv_slots = nullptr;    // [M] cache rows to write
  void* qbuf = nullptr;             // [n_kv][M*G][head_dim] (f16 / bf16)
  void* kcache = nullptr;           // layer base [n_kv][t_max][head_dim]
  void* vcache = nullptr;
  int t_max = 0;
  // EPI_RESID / EPI_SILU: next operand
  float* h = nullptr;               // residual [M][H]
  float* ss_out = nullptr;          // [groups][kSsStride]
  const float* next_norm = nullptr; // norm weight folded into the next operand (null: plain)
  uint32_t* next_frag = nullptr;
  float* next_xsum16 = nullptr;
  float* next_xsum32 = nullptr;
  // Operand column of this op's first output (EPI_SILU; attention ops): under
  // tensor parallelism a rank's slice of the down / O-projection K may start
  // inside a 256-column superblock; the rank then streams whole superblocks
  // and its slice sits at this offset in the wider operand, zeros around it.
  int next_col_off = 0;
  int act_bf16 = 0;                 // operand dtype: 0 f16, 1 bf16
  // Attention ops (FwdOp::kind != OPK_GEMV) use qbuf / kcache / vcache /
  // t_max / head counts above, next_frag / next_xsum* as the O-projection
  // operand they emit, and these:
  const int* attn_step = nullptr;                 // device: [0] prefix length P, [1] total keys
  const unsigned long long* attn_anc = nullptr;   // [M] ancestor bitmask over the new keys
  float* attn_o = nullptr;                        // split partials [n_kv][max_splits][R][hd]
  float* attn_ml = nullptr;                       // [n_kv][max_splits][R][2]
  float attn_scale_log2 = 0.f;                    // log2(e) / sqrt(hd)
  int attn_chunk = 0, attn_max_splits = 0;        // keys per split; splits per KV head
};

// ---- persistent multi-op GEMV kernel -------------------------------------
// One launch runs a schedule of GEMV ops.  Every CTA walks the same op list
// and takes chunks c, c+G, c+2G, ... of each op.  A producer warp streams the
// weight tiles of all its units, across op boundaries, through a TMA ring;
// the activation tile of a stage is only fetched once the op it depends on
// has completed (device-side completion counter), so weight streaming never
// waits on the previous op.
// Op kinds.  Attention ops come last in a launch, after every GEMV op: their
// CTAs stage keys in the weight ring's shared memory once the ring is drained.
//   OPK_ATTN_SPLIT: unit u = (split u / n_kv, KV head u % n_kv) of the split
//     flash decode; waits for the QKV groups of its KV head (dep).
//   OPK_ATTN_COMBINE: unit u = 4 merge items, one per warp; waits for every
//     split unit (dep's done count).
enum OpKind : int { OPK_GEMV = 0, OPK_ATTN_SPLIT = 1, OPK_ATTN_COMBINE = 2 };

struct alignas(16) FwdOp {
  QmvParams q;
  int dep = -1;  // op (index in this launch) whose completion gates this op; -1: the previous kernel
  int kind = OPK_GEMV;
};

// Bit set of weight formats one kernel instantiation handles.
enum FmtSet : int { FS_Q4K = 1, FS_Q5K = 2, FS_Q6K = 4, FS_Q80 = 8, FS_BF16 = 16 };
__host__ __device__ constexpr int fmt_bit(int f) {
  return f == WF_Q4_K ? FS_Q4K : f == WF_Q5_K ? FS_Q5K : f == WF_Q6_K ? FS_Q6K : f == WF_Q8_0 ? FS_Q80 : f == WF_BF16 ? FS_BF16 : 0;
}

constexpr int kMaxLaunchOps = 8;  // ops per forward-kernel launch

struct FwdParams {
  const FwdOp* ops = nullptr;  // device array (16-byte aligned)
  int n_ops = 0;
  int* done = nullptr;         // [n_ops] completion counters, zero at launch
  // Launch attribute (host side): all CTAs co-resident.  Multi-op launches
  // need it: CTA c takes chunks c, c + grid, ... of every op, and a chunk of a
  // later op waits for groups other CTAs produce.
  int cooperative = 0;  // launch attribute (host side): all CTAs co-resident
  unsigned* err = nullptr;
  int l2_ahead = 0;            // stages of this CTA's weights prefetched into L2 ahead of the ring
  // Per-group completion flags [n_ops][flag_stride]: a group's epilogue
  // stores *epoch (this forward's number) into its flag, so a stage of the
  // next op waits only for the groups that produce its K range, not for the
  // whole op.  Null: an op waits for its dependency's `done` count.
  int* gflags = nullptr;
  int flag_stride = 0;
  const unsigned* epoch = nullptr;
  // Consumers that reach the launch's attention ops first signal the next
  // kernel's programmatic launch (griddepcontrol.launch_dependents).
  int trigger_after_gemv = 0;
  // griddepcontrol.launch_dependents at kernel entry (cooperative forward
  // launches only; see fwd_kernel).
  int trigger_at_start = 0;
  // Walk a chunk that starts inside a group from the next group's start and
  // take the piece ending the first group last (see SeqIt in qgemv.cu).
  int rotate = 1;
};

// The instantiation is picked by (format set, nt_for_rows(M)); all ops of
// one launch must share M and have formats inside `fmt_set`.
cudaError_t launch_fwd(const FwdParams& p, int fmt_set, int M, cudaStream_t stream, bool pdl);
// Resident CTAs per SM of the instantiation for `fmt_set` at M <= 8.
int fwd_ctas_per_sm(int fmt_set);
// The format sets instantiated (a model's formats must fit in one).
int fwd_fmt_set_for(int fmt_bits);
// Keys per pass an attention split unit of the forward kernel stages for
// (format set, M rows, head dim, keys per split); below kAttnKeyBlock,
// attention does not fit the instantiation's ring and runs as its own kernels.
int fwd_attn_keys_per_pass(int fmt_set, int M, int hd, int chunk);

// Vocabulary-parallel LM head: holds the stream until *counter >= *target
// (every rank's logits rows of this forward have arrived); bounded wait.
cudaError_t launch_tp_logits_wait(const unsigned long long* counter, const unsigned long long* target, unsigned* err,
                                  cudaStream_t s);

// Repack raw GGUF blocks (device, row-major [N][K/be][bb]) into pair tiles.
cudaError_t launch_repack(const uint8_t* raw, int fmt, int N, int K, uint8_t* tiles, cudaStream_t s);

// ---- embedding gather --------------------------------------------------
struct EmbedParams {
  const uint8_t* table = nullptr;  // raw GGUF rows [V][H]
  int fmt = 0;
  int H = 0, V = 0, M = 0;
  const int* tokens = nullptr;     // [M]
  float* h = nullptr;              // [M][H]
  float* ss_out = nullptr;         // [H/128][kSsStride]
  const float* norm = nullptr;     // first layer's attn_norm
  uint32_t* frag = nullptr;
  float* xsum16 = nullptr;
  float* xsum32 = nullptr;
  int act_bf16 = 0;
  unsigned* err = nullptr;
};
cudaError_t launch_embed(const EmbedParams& p, int nt, cudaStream_t s, bool pdl);

// ---- attention ----------------------------------------------------------
struct AttnParams {
  const void* q = nullptr;         // [n_kv][R][hd], R = M*G, row r = m*G + g
  const void* kcache = nullptr;    // layer base [n_kv][t_max][hd]
  const void* vcache = nullptr;
  int n_kv = 0, G = 0, hd = 0, M = 0, t_max = 0;
  const int* step = nullptr;       // device: [0] = prefix length P, [1] = total keys P + n
  const unsigned long long* anc = nullptr;  // [M] ancestor bitmask over the n new keys
  float scale_log2 = 0.f;          // log2(e) / sqrt(hd)
  int chunk = 64;                  // keys per split (aligned to absolute positions)
  int max_splits = 0;
  float* part_o = nullptr;         // [n_kv][max_splits][R][hd]
  float* part_ml = nullptr;        // [n_kv][max_splits][R][2]
  // combine output: O-proj operand fragments
  uint32_t* frag = nullptr;
  float* xsum16 = nullptr;
  float* xsum32 = nullptr;
  int col_off = 0;                 // operand column of head 0, column 0 (QmvParams::next_col_off)
  int act_bf16 = 0;
  unsigned* err = nullptr;
};
cudaError_t launch_attention(const AttnParams& p, int nt, cudaStream_t s, bool pdl);
// Keys per online-softmax step of a split; a split's chunk is a multiple.
constexpr int kAttnKeyBlock = 32;
// Merge items for R = M*G rows: one warp per (KV head, row, 32 head columns).
__host__ __device__ constexpr int attn_combine_items(int n_kv, int R, int hd) { return n_kv * R * (hd / 32); }

// ---- KV reorder (commit accepted path) -----------------------------------
// src_rows/dst_rows: device int[n]; tmp: device scratch of layers*2*n_kv*n*hd halves.
cudaError_t launch_kv_gather(void* kcache, void* vcache, int layers, int n_kv, int t_max, int hd,
                             const int* src_rows, const int* dst_rows, int n, void* tmp, cudaStream_t s);

// ---- plain f32 activations -> GEMV operand (fragments + column sums) ------
cudaError_t launch_make_operand(const float* x, int M, int K, int nt, uint32_t* frag, float* xsum16, float* xsum32,
                                int bf16, cudaStream_t s);

// ---- final hidden rows (for hidden-state outputs) ------------------------
cudaError_t launch_final_hidden(const float* h, const float* ss, int groups, float inv_dim, float eps,
                                const float* norm, int M, int H, float* out, cudaStream_t s);

// ---- acceptance helpers ---------------------------------------------------
// ---- rejection-sampling acceptance (accept.cu) ----------------------------
enum RejError : int { REJ_OK = 0, REJ_ERR_SOFTMAX = 1, REJ_ERR_ADJUSTED = 2, REJ_ERR_UNIFORMS = 3, REJ_ERR_DISTRIBUTION = 4 };
struct RejStep {
  int k = 0, n_uniforms = 0, budget = 1, pad = 0;
  int drafts[kMaxRows];
  float uniforms[kMaxRows + 1];
};
// rows: [k+1][V] target logits, overwritten with the target probabilities;
// q: [k][V] draft probabilities; r: [V] scratch; out: [4 + kMaxRows] ints,
// zero at launch: n_commits, uniforms used, status (RejError), -, commits.
cudaError_t launch_rejection(float* rows, const float* q, float* r, const RejStep* st, int k, int V,
                             float temperature, int* out, cudaStream_t s);

// ---- typical acceptance over a tree forward (accept.cu) --------------------
struct TypicalTree {
  int n = 0;
  float epsilon = 0.f, delta = 0.f;
  uint32_t tok[kMaxRows];
  int32_t par[kMaxRows];
};
// rows: [n][V] node logits (unchanged).  accept[i] (1 <= i < n) = 1 when
// node i's token passes the typical rule against its parent's row, else 0.
cudaError_t launch_typical_accept(const float* rows, int V, const TypicalTree& t, int* accept, cudaStream_t s);

// Per-row argmax (first-max tie break).  slots / counters: kMaxRows each,
// zero before the first call; every call leaves them zero again.
cudaError_t launch_row_argmax(const float* logits, int rows, int V, int* out_idx, float* out_val,
                              unsigned long long* slots, int* counters, cudaStream_t s);

// Per-row top-k (k <= kMaxTopK): ids[rows][k], vals[rows][k] in descending
// value order, ties by ascending index (methods/medusa.rs:477-487); part:
// scratch of rows * kTopKMaxChunks * k keys.  V <= kTopKMaxChunks * 4096.
constexpr int kMaxTopK = 64;
constexpr int kTopKMaxChunks = 64;
cudaError_t launch_row_topk(const float* logits, int rows, int V, int k, unsigned long long* part, int* ids,
                            float* vals, cudaStream_t s);

// ---- EAGLE draft block glue (methods/eagle.rs:390-427) -------------------
cudaError_t launch_eagle_concat(const uint8_t* table, int fmt, int H, int V, const int* tok, const float* hidden,
                                float* x2, unsigned* err, cudaStream_t s);
cudaError_t launch_eagle_resid_norm(const float* t, const float* h, const float* w, int H, float eps, float* h2,
                                    float* xn, cudaStream_t s);
cudaError_t launch_eagle_add(const float* a, const float* b, float* out, int n, cudaStream_t s);
cudaError_t launch_row_lse(const float* x, int V, float* out, cudaStream_t s);
// Medusa residual block update: out = x + SiLU(y) (methods/medusa.rs:571-575).
cudaError_t launch_medusa_res(const float* x, const float* y, float* out, int n, cudaStream_t s);

// ---- synthetic weight generation (seeded N(0, sigma) then quantized) -------
cudaError_t launch_synth_quant(uint8_t* raw, int fmt, int rows, int K, uint64_t seed, float sigma,
                               int row_offset, cudaStream_t s);
cudaError_t launch_synth_vec(float* out, int n, uint64_t seed, float base, float sigma, cudaStream_t s);

}  // namespace specb200
