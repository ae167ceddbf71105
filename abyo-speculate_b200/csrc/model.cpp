// Host runtime and C ABI of the verify-step backend.
//
// Mirrors the observable protocol of the reference decoders:
//   crates/speculate/src/model/quantized_llama.rs (LlamaQuantDecoder)
//   crates/speculate/src/model/quantized_qwen2.rs (Qwen2QuantDecoder)
//   crates/speculate/src/model/llama.rs           (BF16 LlamaDecoder)
// with history / cache_len / cached-last-logits bookkeeping identical to
// theirs, and the model math of quantized_llama_local.rs /
// quantized_qwen2_local.rs / llama_local.rs executed by this library's CUDA
// kernels (qgemv.cu, attention.cu, misc.cu).
#include "model.h"

#include <math.h>

#include <cmath>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <memory>
#include <new>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/spec_b200.h"
#include "gguf.h"

using namespace specb200;

namespace specb200 {

int choose_chunks(int stages, int resident_ctas) {
  int c = resident_ctas;
  if (const char* env = getenv("SPEC_B200_CHUNKS")) {
    const int v = atoi(env);
    if (v > 0) c = v;
  }
  return std::max(1, std::min(c, stages));
}

}  // namespace specb200

namespace {

thread_local std::string g_load_error;

std::string cuda_msg(cudaError_t e, const char* what) {
  return std::string(what) + ": " + cudaGetErrorString(e);
}

int gcd_int(int a, int b) { return b == 0 ? a : gcd_int(b, a % b); }

uint16_t f2bf_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

float bf_round(float f) {
  uint32_t u = (uint32_t)f2bf_bits(f) << 16;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

}  // namespace

struct EagleHead;  // the EAGLE draft block attached to a target (spec_eagle_*)
struct MedusaHeads;  // Medusa draft heads attached to a target (spec_medusa_*)

struct spec_model {
  ModelCfg cfg;
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  std::string err;
  bool use_graphs = true;

  std::vector<Layer> layers;
  Mat lm;
  uint8_t* embed_raw = nullptr;
  int embed_fmt = 0;
  float* out_norm = nullptr;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;

  int t_max = 0;
  void* kcache = nullptr;
  void* vcache = nullptr;
  size_t kv_layer_elems = 0;

  float* h = nullptr;
  float* ss = nullptr;
  uint32_t* xa = nullptr;
  float* xa16 = nullptr;
  float* xa32 = nullptr;
  uint32_t* xb = nullptr;
  float* xb16 = nullptr;
  float* xb32 = nullptr;
  uint32_t* xc = nullptr;
  float* xc16 = nullptr;
  float* xc32 = nullptr;
  void* qbuf = nullptr;
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int attn_chunk = 64, attn_max_splits = 1;
  float* gemv_part = nullptr;
  int* counters = nullptr;
  size_t part_set = 0;   // floats per partial set (two sets)
  int counter_set = 0;   // counters per set (two sets); also the flag stride
  float* logits = nullptr;
  float* last_row = nullptr;
  float* hidden_out = nullptr;
  float* collect = nullptr;
  unsigned* err_dev = nullptr;
  StepDev* step_dev = nullptr;
  StepDev* step_host = nullptr;
  float* logits_host = nullptr;
  float* hidden_host = nullptr;
  unsigned* err_host = nullptr;
  int* idx_dev = nullptr;
  int* idx_host = nullptr;
  void* kv_tmp = nullptr;
  int* argmax_dev = nullptr;
  unsigned long long* argmax_slots = nullptr;  // row argmax scratch (self-clearing)
  std::shared_ptr<EagleHead> eagle;            // spec_eagle_attach*: device memory owned via dalloc
  std::shared_ptr<MedusaHeads> medusa;         // spec_medusa_attach*: device memory owned via dalloc
  // A tree over kMaxRows nodes leaves only its last chunk's KV rows in the
  // tree window: tree_window lists that chunk's nodes in slot order, for the
  // tree whose signature is tree_window_sig (0: no such tree; every forward
  // clears it).
  std::vector<int> tree_window;
  uint64_t tree_window_sig = 0;
  unsigned long long* topk_part = nullptr;     // row top-k scratch (allocated on first use)
  int* topk_ids = nullptr;
  float* topk_vals = nullptr;
  float* rej_q = nullptr;                      // [kMaxRows-1][V] draft probabilities
  float* rej_q_host = nullptr;                 // pinned staging for rej_q
  float* rej_r = nullptr;                      // [V] adjusted distribution
  RejStep* rej_step_dev = nullptr;
  RejStep* rej_step_host = nullptr;            // pinned
  int* rej_out_dev = nullptr;                  // [4 + kMaxRows]
  int* rej_out_host = nullptr;                 // pinned
  int* argmax_counters = nullptr;
  int* argmax_host = nullptr;
  float* op_in = nullptr;  // f32 staging for apply_lm_head

  std::vector<uint32_t> history;
  int cache_len = 0;
  bool last_valid = false;

  struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    int runs = 0;
  };
  std::map<int, GraphEntry> graphs;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  std::vector<void*> dev_allocs;
  std::vector<void*> host_allocs;
  int64_t weight_bytes = 0;
  int fmt_bits = 0;  // formats present in the model's matrices
  int fmt_set = 0;   // forward-kernel instantiation covering them

  // Device op schedules, one per (rows, flags) forward shape.
  struct Schedule {
    FwdOp* ops = nullptr;
    int* done = nullptr;
    int n_ops = 0;
    std::vector<std::pair<int, int>> launches;  // [begin, end) op slices, one per fwd launch
    std::vector<int64_t> launch_bytes;
    std::vector<FwdOp> host_ops;
    FwdOp* solo = nullptr;  // the same ops with dep = -1, for one-op launches
    int* gflags = nullptr;  // [n_ops][flag_stride] per-group completion flags
    bool fused_attn = false;  // attention runs as ops of the forward kernel
  };
  std::map<int, Schedule> schedules;
  int tp_rank = 0, tp_size = 1;     // tensor-parallel position (1 = whole model on this GPU)
  // K of the O-projection and down matrices as this rank streams them, and
  // where the rank's own columns start inside that window.  Without tensor
  // parallelism: the whole K at offset 0.  With it, a rank's column slice
  // that does not start and end on 256-column superblocks is widened to whole
  // superblocks; the extra columns meet zero activations.
  int o_kwin = 0, o_koff = 0, d_kwin = 0, d_koff = 0;
  // Tensor-parallel receive buffer (exported to the other ranks by CUDA IPC):
  // two sets (o, down), each [tp_size][groups][kTpSlot] flagged 8-byte words.
  uint8_t* tp_buf = nullptr;
  size_t tp_set_bytes = 0;
  void** tp_ptrs_dev = nullptr;     // [set][rank] device pointers to every rank's sets
  // Vocabulary-parallel LM head: this rank owns head rows [lm_row0, lm_row0 +
  // lm.N) of lm_groups_total 128-row groups.  Its logits buffer and arrival
  // counter live in tp_buf (so peers can write them); tp_out_peers_dev[r] is
  // rank r's logits buffer offset to this rank's first row, and
  // tp_out_counters_dev[r] rank r's counter.
  int lm_row0 = 0;
  int lm_groups_total = 0;
  size_t tp_logits_off = 0, tp_counter_off = 0;
  unsigned long long* tp_counter = nullptr;
  float** tp_out_peers_dev = nullptr;
  unsigned long long** tp_out_counters_dev = nullptr;
  unsigned long long logits_forwards = 0;  // forwards with logits (the same count on every rank)
  unsigned epoch = 0;               // forwards run (the same count on every tensor-parallel rank)
  std::vector<void*> tp_peer_bases; // opened IPC mappings (closed at free)
  bool tp_connected = false;
  int l2_ahead = 0;                 // weight stages each CTA prefetches into L2 ahead of its ring (SPEC_B200_L2_AHEAD)
  bool use_pdl = true;              // programmatic dependent launch between forward kernels
  bool fused_attn = false;          // attention as ops of the forward kernel (else its own kernels)
  bool attn_trigger = true;         // a launch's attention tail overlaps the next launch (PDL trigger)
  bool attn_kernels_pdl = true;     // programmatic launch of the standalone attention kernels
  bool coop = true;                 // multi-op forward launches are cooperative (SPEC_B200_NO_COOP clears)
  bool rotate = true;               // chunk walks take a group's tail piece last (SPEC_B200_NO_ROTATE clears)
  bool early_trigger = true;        // cooperative forward launches trigger dependents at entry (SPEC_B200_NO_EARLY_TRIGGER)
  FwdOp* single_op = nullptr;       // device slot for one-op launches
  FwdOp* single_op_host = nullptr;  // pinned staging
  int* single_done = nullptr;

  ~spec_model() {
    DeviceGuard dg_(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto& kv : graphs)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    for (void* p : tp_peer_bases) cudaIpcCloseMemHandle(p);
    for (void* p : dev_allocs) cudaFree(p);
    for (void* p : host_allocs) cudaFreeHost(p);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
  }

  int fail(int code, const std::string& msg) {
    err = msg;
    return code;
  }

  template <class T>
  cudaError_t dalloc(T** p, size_t bytes) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) return e;
    dev_allocs.push_back(q);
    *p = static_cast<T*>(q);
    // Zeroed before returning: the synchronous uploads that often follow run
    // on the legacy stream, which is not ordered after this non-blocking one.
    // (Never called during stream capture: graphs are captured only after a
    // first eager forward has made every buffer.)
    e = cudaMemsetAsync(q, 0, bytes ? bytes : 16, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e;
  }
  // Host -> device copy that has landed when it returns.  A plain cudaMemcpy
  // from pageable memory may return before its DMA completes, and kernels on
  // this non-blocking stream are not ordered after the legacy stream.
  cudaError_t upload(void* dst, const void* src, size_t bytes) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e;
  }
  template <class T>
  cudaError_t halloc(T** p, size_t bytes) {
    void* q = nullptr;
    cudaError_t e = cudaMallocHost(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) return e;
    host_allocs.push_back(q);
    memset(q, 0, bytes ? bytes : 16);
    *p = static_cast<T*>(q);
    return cudaSuccess;
  }
};

namespace {

int kv_elem_bytes(const ModelCfg&) { return 2; }

// ---------------------------------------------------------------------------
// Weight building
// ---------------------------------------------------------------------------

// Copies `rows` raw rows of `row_bytes` from src (host or device) into a
// device destination with an optional destination pitch (for interleaving).
cudaError_t copy_rows(void* dst, size_t dst_pitch, const Part& p, size_t row_bytes, int row0, int rows,
                      cudaStream_t s) {
  const uint8_t* src = p.src + (size_t)row0 * row_bytes;
  const cudaMemcpyKind kind = p.on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (dst_pitch == row_bytes) return cudaMemcpyAsync(dst, src, (size_t)rows * row_bytes, kind, s);
  return cudaMemcpy2DAsync(dst, dst_pitch, src, row_bytes, row_bytes, rows, kind, s);
}

// Build a fused matrix from parts (all of K columns).  interleave64 fuses
// exactly two same-format parts as [a 64 rows | b 64 rows] per 128-row group
// (the gate/up layout consumed by the SiLU epilogue).
int build_mat(spec_model* m, const std::vector<Part>& parts, int K, bool interleave64, Mat& out) {
  // Format runs -> segments.
  struct Run {
    int fmt;
    std::vector<int> idx;
    int rows;
  };
  std::vector<Run> runs;
  for (int i = 0; i < (int)parts.size(); ++i) {
    if (runs.empty() || runs.back().fmt != parts[i].fmt || interleave64) {
      if (interleave64 && !runs.empty()) {
        if (runs.back().fmt != parts[i].fmt) return m->fail(SPEC_ERR_UNSUPPORTED, "gate/up formats differ");
        runs.back().idx.push_back(i);
        runs.back().rows += parts[i].rows;
        continue;
      }
      runs.push_back({parts[i].fmt, {i}, parts[i].rows});
    } else {
      runs.back().idx.push_back(i);
      runs.back().rows += parts[i].rows;
    }
  }
  if (runs.size() > 2) return m->fail(SPEC_ERR_UNSUPPORTED, "more than two weight formats in one fused matrix");
  out.K = K;
  out.N = 0;
  int64_t total = 0;
  for (auto& r : runs) {
    if (fmt_tile_bytes(r.fmt) == 0)
      return m->fail(SPEC_ERR_UNSUPPORTED, "unsupported weight format " + std::to_string(r.fmt));
    if (K % fmt_kt(r.fmt)) return m->fail(SPEC_ERR_UNSUPPORTED, "K not a multiple of the tile width");
    if (r.rows % kGroupRows) return m->fail(SPEC_ERR_UNSUPPORTED, "segment rows not a multiple of 128");
    total += (int64_t)(r.rows / 16) * (K / fmt_kt(r.fmt)) * fmt_tile_bytes(r.fmt);
    out.N += r.rows;
  }
  cudaError_t e = m->dalloc(&out.tiles, (size_t)total);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "weight alloc"));
  out.bytes = total;
  m->weight_bytes += total;
  int64_t off = 0;
  int kgcd = 0;
  for (size_t si = 0; si < runs.size(); ++si) {
    const Run& r = runs[si];
    const size_t row_bytes = (size_t)(K / fmt_block_elems(r.fmt)) * fmt_block_bytes(r.fmt);
    uint8_t* staging = nullptr;
    e = cudaMalloc(&staging, row_bytes * r.rows);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "staging alloc"));
    if (interleave64) {
      const Part& a = parts[r.idx[0]];
      const Part& b = parts[r.idx[1]];
      if (a.rows != b.rows || a.rows % 64) {
        cudaFree(staging);
        return m->fail(SPEC_ERR_UNSUPPORTED, "gate/up shapes differ");
      }
      e = copy_rows(staging, 128 * row_bytes, a, 64 * row_bytes, 0, a.rows / 64, m->stream);
      if (e == cudaSuccess)
        e = copy_rows(staging + 64 * row_bytes, 128 * row_bytes, b, 64 * row_bytes, 0, b.rows / 64, m->stream);
    } else {
      size_t o = 0;
      for (int pi : r.idx) {
        e = copy_rows(staging + o, row_bytes, parts[pi], row_bytes, 0, parts[pi].rows, m->stream);
        if (e != cudaSuccess) break;
        o += row_bytes * parts[pi].rows;
      }
    }
    if (e == cudaSuccess) e = launch_repack(staging, r.fmt, r.rows, K, out.tiles + off, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    cudaFree(staging);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "weight upload/repack"));
    WSeg& sg = out.seg[si];
    sg.w = out.tiles + off;
    sg.fmt = r.fmt;
    sg.groups = r.rows / kGroupRows;
    sg.k_tiles = K / fmt_kt(r.fmt);
    kgcd = kgcd ? gcd_int(kgcd, sg.k_tiles) : sg.k_tiles;
    off += (int64_t)(r.rows / 16) * sg.k_tiles * fmt_tile_bytes(r.fmt);
  }
  if (runs.size() == 1) out.seg[1] = WSeg{};
  const int groups = out.seg[0].groups + out.seg[1].groups;
  const int fa = out.seg[0].fmt, fb = out.seg[1].groups ? out.seg[1].fmt : fa;
  const int bits = fmt_bit(fa) | fmt_bit(fb);
  m->fmt_bits |= bits;
  const int set = fwd_fmt_set_for(bits);
  if (!set) return m->fail(SPEC_ERR_UNSUPPORTED, "weight format combination not supported by the forward kernel");
  out.stages = out.seg[0].groups * out.seg[0].k_tiles + out.seg[1].groups * out.seg[1].k_tiles;
  out.chunks = choose_chunks(out.stages, fwd_ctas_per_sm(set) * m->num_sms);
  (void)groups;
  (void)kgcd;
  return SPEC_OK;
}

// ---------------------------------------------------------------------------
// Buffers and tables
// ---------------------------------------------------------------------------
int alloc_runtime(spec_model* m) {
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, F = c.ffn, V = c.vocab, hd = c.head_dim;
  const int G = c.n_heads / c.n_kv;
  cudaError_t e = cudaSuccess;
#define ALLOC(ptr, bytes)                                                  \
  do {                                                                     \
    e = m->dalloc(&(ptr), (bytes));                                        \
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, #ptr)); \
  } while (0)
#define HALLOC(ptr, bytes)                                                 \
  do {                                                                     \
    e = m->halloc(&(ptr), (bytes));                                        \
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, #ptr)); \
  } while (0)
  m->kv_layer_elems = (size_t)c.n_kv * m->t_max * hd;
  ALLOC(m->kcache, m->kv_layer_elems * c.n_layers * kv_elem_bytes(c));
  ALLOC(m->vcache, m->kv_layer_elems * c.n_layers * kv_elem_bytes(c));
  ALLOC(m->h, (size_t)kMaxRows * H * 4);
  const int groups_h = H / kGroupRows;
  // Two sum-of-squares tables: ss0 = residual after embed / after each down
  // projection, ss1 = after each o-projection (each residual epilogue scales
  // its emitted operand by the other table's rinv).
  ALLOC(m->ss, (size_t)2 * groups_h * kSsStride * 4);
  // O-projection and down operands span the K windows the rank streams; the
  // columns outside its own slice are cleared for each forward's layout
  // (zero_window_edges).
  const int Kq = m->o_kwin, Kd = m->d_kwin;
  auto frag_bytes = [](int K) { return (size_t)K * kMaxRows * 2; };
  ALLOC(m->xa, frag_bytes(H));
  ALLOC(m->xa16, (size_t)(H / 16) * kMaxRows * 4);
  ALLOC(m->xa32, (size_t)(H / 32) * kMaxRows * 4);
  ALLOC(m->xb, frag_bytes(Kq));
  ALLOC(m->xb16, (size_t)(Kq / 16) * kMaxRows * 4);
  ALLOC(m->xb32, (size_t)(Kq / 32) * kMaxRows * 4);
  ALLOC(m->xc, frag_bytes(Kd));
  ALLOC(m->xc16, (size_t)(Kd / 16) * kMaxRows * 4);
  ALLOC(m->xc32, (size_t)(Kd / 32) * kMaxRows * 4);
  ALLOC(m->qbuf, (size_t)c.n_heads * kMaxRows * hd * 2);
  // Keys per attention split (fixed per model: splits are aligned to absolute
  // key positions, which keeps every row's arithmetic independent of M).
  // Long contexts take larger splits (fewer partials to merge).
  m->attn_chunk = m->t_max <= 8192 ? 128 : 256;
  if (const char* env = getenv("SPEC_B200_ATTN_CHUNK")) {  // tuning override: 64, 128 or 256 keys
    const int v = atoi(env);
    if (v == 64 || v == 128 || v == 256) m->attn_chunk = v;
  }
  m->attn_max_splits = (m->t_max + m->attn_chunk - 1) / m->attn_chunk;
  const size_t R = (size_t)kMaxRows * G;
  ALLOC(m->part_o, (size_t)c.n_kv * m->attn_max_splits * R * hd * 4);
  ALLOC(m->part_ml, (size_t)c.n_kv * m->attn_max_splits * R * 2 * 4);
  size_t part = 0;
  int max_groups = 0;
  auto acc_mat = [&](const Mat& mt) {
    const int g = mt.seg[0].groups + mt.seg[1].groups;
    max_groups = std::max(max_groups, g);
    part = std::max(part, (size_t)partial_slots(mt) * kGroupRows * kMaxRows);
  };
  for (auto& L : m->layers) {
    acc_mat(L.qkv);
    acc_mat(L.o);
    acc_mat(L.gu);
    acc_mat(L.down);
  }
  acc_mat(m->lm);
  // Two sets of split-K partials and arrival counters, used by alternate ops
  // of a launch: with per-group dependencies, op i+1 can start while op i
  // still reduces; op i+2 starts only after op i is complete.
  m->part_set = part;
  m->counter_set = max_groups;
  ALLOC(m->gemv_part, 2 * part * 4);
  ALLOC(m->counters, (size_t)2 * max_groups * 4);
  if (m->tp_size > 1) {
    // [o set][down set][logits kMaxRows x V][arrival counter]: one exported
    // allocation, the same layout on every rank.
    auto up256 = [](size_t v) { return (v + 255) / 256 * 256; };
    m->tp_set_bytes = up256((size_t)m->tp_size * groups_h * kTpSlot * 8);
    m->tp_logits_off = 2 * m->tp_set_bytes;
    m->tp_counter_off = m->tp_logits_off + up256((size_t)kMaxRows * V * 4);
    ALLOC(m->tp_buf, m->tp_counter_off + 256);
    ALLOC(m->tp_ptrs_dev, (size_t)2 * m->tp_size * sizeof(void*));
    ALLOC(m->tp_out_peers_dev, (size_t)m->tp_size * sizeof(float*));
    ALLOC(m->tp_out_counters_dev, (size_t)m->tp_size * sizeof(unsigned long long*));
    m->logits = reinterpret_cast<float*>(m->tp_buf + m->tp_logits_off);
    m->tp_counter = reinterpret_cast<unsigned long long*>(m->tp_buf + m->tp_counter_off);
  } else {
    ALLOC(m->logits, (size_t)kMaxRows * V * 4);
  }
  ALLOC(m->last_row, (size_t)V * 4);
  ALLOC(m->hidden_out, (size_t)kMaxRows * H * 4);
  ALLOC(m->err_dev, 16);
  ALLOC(m->step_dev, sizeof(StepDev));
  ALLOC(m->idx_dev, 4 * (size_t)(m->t_max + 64) * 2);
  ALLOC(m->kv_tmp, (size_t)c.n_layers * 2 * c.n_kv * kMaxRows * hd * 2);
  ALLOC(m->argmax_dev, kMaxRows * 4);
  ALLOC(m->argmax_slots, kMaxRows * 8);
  ALLOC(m->rej_q, (size_t)(kMaxRows - 1) * V * 4);
  HALLOC(m->rej_q_host, (size_t)(kMaxRows - 1) * V * 4);
  ALLOC(m->rej_r, (size_t)V * 4);
  ALLOC(m->rej_step_dev, sizeof(RejStep));
  HALLOC(m->rej_step_host, sizeof(RejStep));
  ALLOC(m->rej_out_dev, (4 + kMaxRows) * 4);
  HALLOC(m->rej_out_host, (4 + kMaxRows) * 4);
  ALLOC(m->argmax_counters, kMaxRows * 4);
  ALLOC(m->op_in, (size_t)kMaxRows * H * 4);
  HALLOC(m->step_host, sizeof(StepDev));
  HALLOC(m->logits_host, (size_t)kMaxRows * V * 4);
  HALLOC(m->hidden_host, (size_t)kMaxRows * H * 4);
  HALLOC(m->err_host, 16);
  HALLOC(m->idx_host, 4 * (size_t)(m->t_max + 64) * 2);
  HALLOC(m->argmax_host, kMaxRows * 4);
#undef ALLOC
#undef HALLOC
  e = cudaEventCreate(&m->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&m->ev1);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "events"));
  return SPEC_OK;
}

// RoPE tables exactly as precomput_freqs_cis (quantized_llama_local.rs:189-205):
// theta_i = 1 / base^(2i/d) in f32, angle = pos * theta_i (single f32
// product), cos/sin in f32.  Llama-3 frequency scaling follows
// llama_local.rs:47-75; the BF16 model casts the tables to bf16 (:95-96).
int build_rope(spec_model* m) {
  const ModelCfg& c = m->cfg;
  const int half = c.head_dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(c.rope_theta, (float)(2 * i) / (float)c.head_dim);
  if (c.rope_scaled) {
    const float pi = 3.14159265358979323846f;
    const float low_wavelen = (float)c.rs_orig / c.rs_low;
    const float high_wavelen = (float)c.rs_orig / c.rs_high;
    for (int i = 0; i < half; ++i) {
      const float freq = inv[i];
      const float wavelen = 2.f * pi / freq;
      if (wavelen < high_wavelen) {
      } else if (wavelen > low_wavelen) {
        inv[i] = freq / c.rs_factor;
      } else {
        const float smooth = ((float)c.rs_orig / wavelen - c.rs_low) / (c.rs_high - c.rs_low);
        inv[i] = (1.f - smooth) * freq / c.rs_factor + smooth * freq;
      }
    }
  }
  const size_t n = (size_t)m->t_max * half;
  std::vector<float> cs(n), sn(n);
  for (int p = 0; p < m->t_max; ++p)
    for (int i = 0; i < half; ++i) {
      const float a = (float)p * inv[i];
      float cv = cosf(a), sv = sinf(a);
      if (c.rope_tables_bf16) {
        cv = bf_round(cv);
        sv = bf_round(sv);
      }
      cs[(size_t)p * half + i] = cv;
      sn[(size_t)p * half + i] = sv;
    }
  cudaError_t e = m->dalloc(&m->rope_cos, n * 4);
  if (e == cudaSuccess) e = m->dalloc(&m->rope_sin, n * 4);
  if (e == cudaSuccess) e = m->upload(m->rope_cos, cs.data(), n * 4);
  if (e == cudaSuccess) e = m->upload(m->rope_sin, sn.data(), n * 4);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "rope tables"));
  return SPEC_OK;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
enum : int { F_LOGITS = 1, F_HIDDEN = 2 };

QmvParams base_params(spec_model* m, const Mat& mt, int M) {
  QmvParams p;
  p.seg[0] = mt.seg[0];
  p.seg[1] = mt.seg[1];
  p.n_rows = mt.N;
  p.K = mt.K;
  p.stages = mt.stages;
  p.chunks = mt.chunks;
  p.M = M;
  p.part = m->gemv_part;
  p.counters = m->counters;
  p.err = m->err_dev;
  p.act_bf16 = m->cfg.bf16 ? 1 : 0;
  return p;
}

struct ProfRec {
  std::vector<cudaEvent_t> ev;  // ev[0] before the first kernel, ev[i+1] after kernel i
  std::vector<int> kind;
  std::vector<int64_t> bytes;
};

// Kernel kinds reported by spec_profile_forward.
enum : int { K_EMBED = 0, K_ATTN = 2 };

cudaError_t prof_mark(ProfRec* pr, cudaStream_t s, int kind, int64_t bytes) {
  if (!pr) return cudaSuccess;
  cudaEvent_t e;
  cudaError_t err = cudaEventCreate(&e);
  if (err != cudaSuccess) return err;
  pr->ev.push_back(e);
  pr->kind.push_back(kind);
  pr->bytes.push_back(bytes);
  return cudaEventRecord(e, s);
}

// Kernel kinds reported by spec_profile_forward (K_FWD: one persistent
// multi-op GEMV launch).
enum : int { K_FWD = 8 };

// Points a row-parallel op's epilogue at its tensor-parallel receive set.
void set_tp(spec_model* m, QmvParams& p, int layer, int set) {
  if (m->tp_size <= 1) return;
  p.tp_size = m->tp_size;
  p.tp_rank = m->tp_rank;
  p.tp_tag = 2 * layer + set;
  p.tp_epoch = &m->step_dev->epoch;
  p.tp_recv = reinterpret_cast<unsigned long long* const*>(m->tp_ptrs_dev + (size_t)set * m->tp_size);
  p.tp_recv_local = reinterpret_cast<const unsigned long long*>(m->tp_buf + set * m->tp_set_bytes);
}

// The two sum-of-squares tables (see alloc_runtime).
float* ss0(spec_model* m) { return m->ss; }
float* ss1(spec_model* m) { return m->ss + (size_t)(m->cfg.hidden / kGroupRows) * kSsStride; }

// GEMV op descriptors of one layer (QKV; O; gate/up; down) for M rows.
FwdOp op_qkv(spec_model* m, int l, int M) {
  const ModelCfg& c = m->cfg;
  const Layer& L = m->layers[l];
  FwdOp o;
  QmvParams& p = o.q;
  p = base_params(m, L.qkv, M);
  p.xfrag = m->xa;
  p.xsum16 = m->xa16;
  p.xsum32 = m->xa32;
  p.ss_in = ss0(m);
  p.ss_pre = l > 0 ? ss1(m) : nullptr;  // layer 0's operand comes from embed, unscaled
  p.ss_groups = c.hidden / kGroupRows;
  p.ss_inv_dim = 1.f / (float)c.hidden;
  p.eps = c.eps;
  p.epi = EPI_QKV;
  p.bias = L.bqkv;
  p.n_q_heads = c.n_heads;
  p.n_kv_heads = c.n_kv;
  p.head_dim = c.head_dim;
  p.rope_interleaved = c.rope_interleaved ? 1 : 0;
  p.rope_cos = m->rope_cos;
  p.rope_sin = m->rope_sin;
  p.positions = m->step_dev->positions;
  p.kv_slots = m->step_dev->slots;
  p.qbuf = m->qbuf;
  p.kcache = static_cast<uint8_t*>(m->kcache) + (size_t)l * m->kv_layer_elems * 2;
  p.vcache = static_cast<uint8_t*>(m->vcache) + (size_t)l * m->kv_layer_elems * 2;
  p.t_max = m->t_max;
  return o;
}
// Layer l's attention as ops of the forward kernel, after its QKV op:
// OPK_ATTN_SPLIT (one unit per (split, KV head)) and OPK_ATTN_COMBINE (four
// merge items per unit, emitting the O-projection operand).
FwdOp op_attn(spec_model* m, int l, int M, int kind) {
  const ModelCfg& c = m->cfg;
  FwdOp o;
  o.kind = kind;
  QmvParams& p = o.q;
  p.M = M;
  p.err = m->err_dev;
  p.act_bf16 = c.bf16 ? 1 : 0;
  p.n_q_heads = c.n_heads;
  p.n_kv_heads = c.n_kv;
  p.head_dim = c.head_dim;
  p.qbuf = m->qbuf;
  p.kcache = static_cast<uint8_t*>(m->kcache) + (size_t)l * m->kv_layer_elems * 2;
  p.vcache = static_cast<uint8_t*>(m->vcache) + (size_t)l * m->kv_layer_elems * 2;
  p.t_max = m->t_max;
  p.attn_step = m->step_dev->step;
  p.attn_anc = m->step_dev->anc;
  p.attn_o = m->part_o;
  p.attn_ml = m->part_ml;
  p.attn_scale_log2 = 1.4426950408889634f / sqrtf((float)c.head_dim);
  p.attn_chunk = m->attn_chunk;
  p.attn_max_splits = m->attn_max_splits;
  p.next_frag = m->xb;
  p.next_xsum16 = m->xb16;
  p.next_xsum32 = m->xb32;
  p.next_col_off = m->o_koff;
  const int R = M * (c.n_heads / c.n_kv);
  p.stages = p.chunks = kind == OPK_ATTN_SPLIT
                            ? c.n_kv * m->attn_max_splits
                            : (attn_combine_items(c.n_kv, R, c.head_dim) + kGemvWarps - 1) / kGemvWarps;
  return o;
}

// Whether attention runs inside the forward kernel for M rows: the split
// unit's key / query staging must fit the weight ring of the instantiation.
bool attn_fused(const spec_model* m, int M) {
  if (!m->fused_attn) return false;
  const int hd = m->cfg.head_dim;
  if (hd != 64 && hd != 128) return false;
  return fwd_attn_keys_per_pass(m->fmt_set, M, hd, m->attn_chunk) >= kAttnKeyBlock;
}

FwdOp op_o(spec_model* m, int l, int M) {
  const ModelCfg& c = m->cfg;
  FwdOp o;
  QmvParams& p = o.q;
  p = base_params(m, m->layers[l].o, M);
  p.xfrag = m->xb;
  p.xsum16 = m->xb16;
  p.xsum32 = m->xb32;
  p.epi = EPI_RESID;
  p.h = m->h;
  p.ss_out = ss1(m);
  p.ss_scale = ss0(m);  // residual before this update: embed's or the previous down's
  p.ss_groups = c.hidden / kGroupRows;
  p.ss_inv_dim = 1.f / (float)c.hidden;
  p.eps = c.eps;
  p.next_norm = m->layers[l].ffn_norm;
  p.next_frag = m->xa;
  p.next_xsum16 = m->xa16;
  p.next_xsum32 = m->xa32;
  set_tp(m, p, l, 0);
  return o;
}
FwdOp op_gu(spec_model* m, int l, int M) {
  const ModelCfg& c = m->cfg;
  FwdOp o;
  QmvParams& p = o.q;
  p = base_params(m, m->layers[l].gu, M);
  p.xfrag = m->xa;
  p.xsum16 = m->xa16;
  p.xsum32 = m->xa32;
  p.ss_in = ss1(m);
  p.ss_pre = ss0(m);
  p.ss_groups = c.hidden / kGroupRows;
  p.ss_inv_dim = 1.f / (float)c.hidden;
  p.eps = c.eps;
  p.epi = EPI_SILU;
  p.next_frag = m->xc;
  p.next_xsum16 = m->xc16;
  p.next_xsum32 = m->xc32;
  p.next_col_off = m->d_koff;
  return o;
}
FwdOp op_down(spec_model* m, int l, int M) {
  const ModelCfg& c = m->cfg;
  FwdOp o;
  QmvParams& p = o.q;
  p = base_params(m, m->layers[l].down, M);
  p.xfrag = m->xc;
  p.xsum16 = m->xc16;
  p.xsum32 = m->xc32;
  p.epi = EPI_RESID;
  p.h = m->h;
  p.ss_out = ss0(m);
  p.ss_scale = ss1(m);  // residual before this update: the o-projection's
  p.ss_groups = c.hidden / kGroupRows;
  p.ss_inv_dim = 1.f / (float)c.hidden;
  p.eps = c.eps;
  p.next_norm = (l + 1 < c.n_layers) ? m->layers[l + 1].attn_norm : m->out_norm;
  p.next_frag = m->xa;
  p.next_xsum16 = m->xa16;
  p.next_xsum32 = m->xa32;
  set_tp(m, p, l, 1);
  return o;
}
FwdOp op_lm(spec_model* m, int M, float* out) {
  const ModelCfg& c = m->cfg;
  FwdOp o;
  QmvParams& p = o.q;
  p = base_params(m, m->lm, M);
  p.xfrag = m->xa;
  p.xsum16 = m->xa16;
  p.xsum32 = m->xa32;
  p.ss_in = ss0(m);
  p.ss_pre = ss1(m);
  p.ss_groups = c.hidden / kGroupRows;
  p.ss_inv_dim = 1.f / (float)c.hidden;
  p.eps = c.eps;
  p.epi = EPI_STORE;
  p.out = out + m->lm_row0;  // this rank's rows of the head (all rows without tensor parallelism)
  p.ld_out = c.vocab;
  if (m->tp_size > 1 && out == m->logits) {
    p.out_ranks = m->tp_size;
    p.out_peers = m->tp_out_peers_dev;
    p.out_counters = m->tp_out_counters_dev;
  }
  return o;
}

// The forward's GEMV schedule for (M, flags): launch 0 = [L0.QKV]; launch
// l+1 = [Ll.O, Ll.gate/up, Ll.down, L(l+1).QKV | LM head].  Uploaded once.
int get_schedule(spec_model* m, int M, int flags, spec_model::Schedule** out) {
  const int key = M | (flags << 8);
  auto it = m->schedules.find(key);
  if (it != m->schedules.end()) {
    *out = &it->second;
    return SPEC_OK;
  }
  const ModelCfg& c = m->cfg;
  spec_model::Schedule sc;
  std::vector<FwdOp> ops;
  auto begin_launch = [&]() { sc.launches.push_back({(int)ops.size(), (int)ops.size()}); sc.launch_bytes.push_back(0); };
  auto add = [&](FwdOp o, int64_t bytes) {
    const int first = sc.launches.back().first;
    o.dep = (int)ops.size() == first ? -1 : (int)ops.size() - 1 - first;
    if (o.kind == OPK_GEMV && (((int)ops.size() - first) & 1)) {
      o.q.part += m->part_set;
      o.q.counters += m->counter_set;
    }
    ops.push_back(o);
    sc.launches.back().second = (int)ops.size();
    sc.launch_bytes.back() += bytes;
  };
  if (!m->fmt_set) m->fmt_set = fwd_fmt_set_for(m->fmt_bits);
  sc.fused_attn = attn_fused(m, M);
  auto add_attn = [&](int l) {
    if (!sc.fused_attn) return;
    add(op_attn(m, l, M, OPK_ATTN_SPLIT), 0);
    add(op_attn(m, l, M, OPK_ATTN_COMBINE), 0);
  };
  begin_launch();
  add(op_qkv(m, 0, M), m->layers[0].qkv.bytes);
  add_attn(0);
  for (int l = 0; l < c.n_layers; ++l) {
    begin_launch();
    add(op_o(m, l, M), m->layers[l].o.bytes);
    add(op_gu(m, l, M), m->layers[l].gu.bytes);
    add(op_down(m, l, M), m->layers[l].down.bytes);
    if (l + 1 < c.n_layers) {
      add(op_qkv(m, l + 1, M), m->layers[l + 1].qkv.bytes);
      add_attn(l + 1);
    } else if (flags & F_LOGITS) {
      add(op_lm(m, M, m->logits), m->lm.bytes);
    }
  }
  sc.n_ops = (int)ops.size();
  sc.host_ops = ops;
  cudaError_t e = m->dalloc(&sc.ops, sizeof(FwdOp) * ops.size());
  if (e == cudaSuccess) e = m->dalloc(&sc.done, sizeof(int) * ops.size());
  if (e == cudaSuccess) e = m->dalloc(&sc.gflags, sizeof(int) * ops.size() * m->counter_set);
  if (e == cudaSuccess) e = m->upload(sc.ops, ops.data(), sizeof(FwdOp) * ops.size());
  if (e == cudaSuccess) {
    std::vector<FwdOp> solo = ops;
    for (auto& o : solo) o.dep = -1;
    e = m->dalloc(&sc.solo, sizeof(FwdOp) * solo.size());
    if (e == cudaSuccess)
      e = m->upload(sc.solo, solo.data(), sizeof(FwdOp) * solo.size());
  }
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "schedule upload"));
  auto res = m->schedules.emplace(key, std::move(sc));
  *out = &res.first->second;
  return SPEC_OK;
}

cudaError_t launch_slice(spec_model* m, const spec_model::Schedule& sc, int li, int M, bool pdl) {
  FwdParams fp;
  fp.ops = sc.ops + sc.launches[li].first;
  fp.n_ops = sc.launches[li].second - sc.launches[li].first;
  fp.done = sc.done + sc.launches[li].first;
  // A cooperative launch: every CTA resident, so no CTA waits on a group
  // whose CTA has not started.
  fp.cooperative = (m->coop && fp.n_ops > 1) ? 1 : 0;
  fp.err = m->err_dev;
  fp.l2_ahead = m->l2_ahead;
  fp.gflags = sc.gflags + (size_t)sc.launches[li].first * m->counter_set;
  fp.flag_stride = m->counter_set;
  fp.epoch = &m->step_dev->epoch;
  fp.trigger_after_gemv = (pdl && m->attn_trigger) ? 1 : 0;
  fp.trigger_at_start = (pdl && fp.cooperative && m->early_trigger) ? 1 : 0;
  fp.rotate = m->rotate ? 1 : 0;
  return launch_fwd(fp, m->fmt_set, M, m->stream, pdl);
}

// One GEMV op as its own launch (apply_lm_head, the standalone dequant
// matmul).  The op descriptor goes through pinned staging on the stream.
cudaError_t enqueue_single(spec_model* m, const QmvParams& q, cudaStream_t s) {
  cudaError_t e = cudaSuccess;
  if (!m->single_op) {
    e = m->dalloc(&m->single_op, sizeof(FwdOp));
    if (e == cudaSuccess) e = m->dalloc(&m->single_done, 16);
    if (e == cudaSuccess) e = m->halloc(&m->single_op_host, sizeof(FwdOp));
    if (e != cudaSuccess) return e;
  }
  if (!m->fmt_set) m->fmt_set = fwd_fmt_set_for(m->fmt_bits);
  cudaStreamSynchronize(s);  // the staging slot may still feed a previous copy
  *m->single_op_host = FwdOp{};
  m->single_op_host->q = q;
  m->single_op_host->dep = -1;
  e = cudaMemcpyAsync(m->single_op, m->single_op_host, sizeof(FwdOp), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->single_done, 0, 16, s);
  if (e != cudaSuccess) return e;
  FwdParams fp;
  fp.ops = m->single_op;
  fp.n_ops = 1;
  fp.done = m->single_done;
  fp.err = m->err_dev;
  fp.l2_ahead = m->l2_ahead;
  return launch_fwd(fp, m->fmt_set, q.M, s, false);
}

// Op q of a schedule as its own launch (used when every layer's output is
// collected between the ops of a slice).
cudaError_t launch_solo(spec_model* m, spec_model::Schedule* sc, int q, int M, cudaStream_t s) {
  FwdParams fp;
  fp.ops = sc->solo + q;
  fp.n_ops = 1;
  fp.done = sc->done + q;
  fp.err = m->err_dev;
  fp.l2_ahead = m->l2_ahead;
  return launch_fwd(fp, m->fmt_set, M, s, false);
}

// Under tensor parallelism a rank's O-projection / down operand spans a
// window of whole superblocks around its own columns [off, off + len), and
// the columns outside its slice must read as zero.  Where those columns sit
// in memory depends on the operand layout of the forward's row count (n-tiles
// per k-step), so a forward with another row count may have written there:
// each forward clears them for its own layout.  off, len and win are
// multiples of 128 columns (whole k-steps and 32-column sum blocks).
cudaError_t zero_window_edges(uint32_t* frag, float* x16, float* x32, int win, int off, int len, int nt,
                              cudaStream_t s) {
  auto clear = [&](int k0, int k1) -> cudaError_t {
    if (k1 <= k0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(reinterpret_cast<uint8_t*>(frag) + (size_t)(k0 / 16) * nt * 256, 0,
                                    (size_t)(k1 - k0) / 16 * nt * 256, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(x16 + (size_t)(k0 / 16) * 8 * nt, 0, (size_t)(k1 - k0) / 16 * 8 * nt * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(x32 + (size_t)(k0 / 32) * 8 * nt, 0, (size_t)(k1 - k0) / 32 * 8 * nt * 4, s);
    return e;
  };
  cudaError_t e = clear(0, off);
  if (e == cudaSuccess) e = clear(off + len, win);
  return e;
}

cudaError_t enqueue_forward(spec_model* m, int M, int flags, const std::vector<int>* collect,
                            ProfRec* pr = nullptr) {
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, hd = c.head_dim, G = c.n_heads / c.n_kv;
  const int nt = nt_for_rows(M);
  cudaStream_t s = m->stream;
  spec_model::Schedule* sc = nullptr;
  if (get_schedule(m, M, flags, &sc) != SPEC_OK) return cudaErrorMemoryAllocation;
  cudaError_t e = cudaMemcpyAsync(m->step_dev, m->step_host, sizeof(StepDev), cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(sc->done, 0, sizeof(int) * sc->n_ops, s);
  if (e != cudaSuccess) return e;
  if (m->tp_size > 1) {  // c holds this rank's head and FFN counts
    e = zero_window_edges(m->xb, m->xb16, m->xb32, m->o_kwin, m->o_koff, c.n_heads * hd, nt, s);
    if (e == cudaSuccess) e = zero_window_edges(m->xc, m->xc16, m->xc32, m->d_kwin, m->d_koff, c.ffn, nt, s);
    if (e != cudaSuccess) return e;
  }
  EmbedParams ep;
  ep.table = m->embed_raw;
  ep.fmt = m->embed_fmt;
  ep.H = H;
  ep.V = c.vocab;
  ep.M = M;
  ep.tokens = m->step_dev->tokens;
  ep.h = m->h;
  ep.ss_out = m->ss;
  ep.norm = m->layers[0].attn_norm;
  ep.frag = m->xa;
  ep.xsum16 = m->xa16;
  ep.xsum32 = m->xa32;
  ep.act_bf16 = c.bf16 ? 1 : 0;
  ep.err = m->err_dev;
  if (pr) {
    cudaEvent_t e0;
    if ((e = cudaEventCreate(&e0)) != cudaSuccess) return e;
    pr->ev.push_back(e0);
    if ((e = cudaEventRecord(e0, s)) != cudaSuccess) return e;
  }
  const bool pdl = pr == nullptr && m->use_pdl;
  e = launch_embed(ep, nt, s, false);
  if (e != cudaSuccess) return e;
  if ((e = prof_mark(pr, s, K_EMBED, (int64_t)M * H * 8)) != cudaSuccess) return e;
  const int64_t step_keys = (int64_t)m->step_host->step[1];
  // K and V bytes one layer's attention reads (counted in the forward
  // kernel's launch when attention runs inside it).
  const int64_t attn_bytes = step_keys * c.n_kv * hd * 2 * 2;
  const int64_t fused_bytes = sc->fused_attn ? attn_bytes : 0;
  if ((e = launch_slice(m, *sc, 0, M, pdl)) != cudaSuccess) return e;
  if ((e = prof_mark(pr, s, K_FWD, sc->launch_bytes[0] + fused_bytes)) != cudaSuccess) return e;
  for (int l = 0; l < c.n_layers; ++l) {
    if (!sc->fused_attn) {  // attention of layer l as its own kernels
      AttnParams a;
      a.q = m->qbuf;
      a.kcache = static_cast<uint8_t*>(m->kcache) + (size_t)l * m->kv_layer_elems * 2;
      a.vcache = static_cast<uint8_t*>(m->vcache) + (size_t)l * m->kv_layer_elems * 2;
      a.n_kv = c.n_kv;
      a.G = G;
      a.hd = hd;
      a.M = M;
      a.t_max = m->t_max;
      a.step = m->step_dev->step;
      a.anc = m->step_dev->anc;
      a.scale_log2 = 1.4426950408889634f / sqrtf((float)hd);
      a.chunk = m->attn_chunk;
      a.max_splits = m->attn_max_splits;
      a.part_o = m->part_o;
      a.part_ml = m->part_ml;
      a.frag = m->xb;
      a.xsum16 = m->xb16;
      a.xsum32 = m->xb32;
      a.col_off = m->o_koff;
      a.act_bf16 = c.bf16 ? 1 : 0;
      a.err = m->err_dev;
      // 64-key splits launch 512+ small split CTAs.  Chained programmatically
      // ahead of a forward kernel whose CTAs could start before all of them
      // fit, they lost a GEMV group's completion on B200 (a bounded wait
      // fired).  A cooperative forward launch cannot be caught that way;
      // without it they run without the early launch.
      const bool attn_pdl = pdl && m->attn_kernels_pdl && (m->attn_chunk >= 128 || m->coop);
      if ((e = launch_attention(a, nt, s, attn_pdl)) != cudaSuccess) return e;
      if ((e = prof_mark(pr, s, K_ATTN, attn_bytes)) != cudaSuccess) return e;
    }
    if (collect) {
      // Collecting a layer's residual splits the launch after its down-proj.
      bool want = false;
      for (int v : *collect) want |= (v == l);
      if (want) {
        // Run [O, gate/up, down] of this layer as single-op launches so the
        // residual can be copied before the next layer's QKV overwrites it.
        const auto& sl = sc->launches[l + 1];
        for (int q = sl.first; q < sl.first + 3; ++q)
          if ((e = launch_solo(m, sc, q, M, s)) != cudaSuccess) return e;
        for (size_t ci = 0; ci < collect->size(); ++ci)
          if ((*collect)[ci] == l) {
            e = cudaMemcpyAsync(m->collect + ci * (size_t)M * H, m->h, (size_t)M * H * 4, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return e;
          }
        for (int q = sl.first + 3; q < sl.second; ++q)
          if ((e = launch_solo(m, sc, q, M, s)) != cudaSuccess) return e;
        continue;
      }
    }
    if ((e = launch_slice(m, *sc, l + 1, M, pdl)) != cudaSuccess) return e;
    const bool has_attn = sc->fused_attn && l + 1 < c.n_layers;
    if ((e = prof_mark(pr, s, K_FWD, sc->launch_bytes[l + 1] + (has_attn ? attn_bytes : 0))) != cudaSuccess) return e;
  }
  if ((flags & F_LOGITS) && m->tp_size > 1) {
    // Vocabulary-parallel head: every rank's rows must be in this rank's
    // logits before anything reads them.
    e = launch_tp_logits_wait(m->tp_counter, &m->step_dev->logits_target, m->err_dev, s);
    if (e != cudaSuccess) return e;
  }
  if (flags & F_LOGITS) {
    e = cudaMemcpyAsync(m->last_row, m->logits + (size_t)(M - 1) * c.vocab, (size_t)c.vocab * 4,
                        cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
  }
  if (flags & F_HIDDEN) {
    e = launch_final_hidden(m->h, m->ss, H / kGroupRows, 1.f / (float)H, c.eps, m->out_norm, M, H, m->hidden_out, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Runs one forward of M rows described by m->step_host.  Graph-replayed per
// (M, flags) after a first eager run.
// Numbers the forward about to be enqueued: its completion-flag / exchange
// epoch and, with logits under tensor parallelism, the arrival count that
// says every rank's LM-head rows are in.
void begin_step(spec_model* m, int flags) {
  m->step_host->epoch = ++m->epoch;
  if (flags & F_LOGITS) ++m->logits_forwards;
  m->step_host->logits_target = m->logits_forwards * (unsigned long long)m->lm_groups_total;
}

int run_forward(spec_model* m, int M, int flags, const std::vector<int>* collect = nullptr) {
  if (m->tp_size > 1 && !m->tp_connected)
    return m->fail(SPEC_ERR_INVALID, "tensor-parallel handle used before spec_tp_connect");
  m->tree_window_sig = 0;
  begin_step(m, flags);
  cudaError_t e = cudaSuccess;
  const int key = M | (flags << 8);
  const bool graphable = m->use_graphs && collect == nullptr;
  e = cudaEventRecord(m->ev0, m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "event"));
  auto& ge = m->graphs[key];
  if (graphable && ge.exec) {
    e = cudaGraphLaunch(ge.exec, m->stream);
  } else if (graphable && ge.runs >= 1) {
    cudaGraph_t g = nullptr;
    e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const cudaError_t ee = enqueue_forward(m, M, flags, nullptr);
      e = cudaStreamEndCapture(m->stream, &g);
      if (ee != cudaSuccess) e = ee;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&ge.exec, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e == cudaSuccess) e = cudaGraphLaunch(ge.exec, m->stream);
    if (e != cudaSuccess) {
      // Capture unsupported here: fall back to eager launches for good.
      cudaGetLastError();
      if (ge.exec) cudaGraphExecDestroy(ge.exec);
      ge.exec = nullptr;
      m->use_graphs = false;
      e = enqueue_forward(m, M, flags, nullptr);
    }
  } else {
    e = enqueue_forward(m, M, flags, collect);
  }
  ge.runs++;
  if (e == cudaSuccess) e = cudaEventRecord(m->ev1, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->err_host, m->err_dev, 16, cudaMemcpyDeviceToHost, m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "forward launch"));
  return SPEC_OK;
}

int finish(spec_model* m) {
  cudaError_t e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "forward"));
  cudaEventElapsedTime(&m->last_ms, m->ev0, m->ev1);
  if (*m->err_host) {
    const unsigned bits = m->err_host[0], where = m->err_host[1], pos = m->err_host[2], seen = m->err_host[3];
    for (int i = 0; i < 4; ++i) m->err_host[i] = 0;
    cudaMemsetAsync(m->err_dev, 0, 16, m->stream);
    cudaStreamSynchronize(m->stream);
    if (bits & DEV_ERR_MBAR_TIMEOUT) {
      char msg[192];
      snprintf(msg, sizeof msg,
               "a device wait gave up (mbarrier timeout): site %u op %u cta %u, stage/pos %u (0x%x), counter %d",
               where & 0xffu, (where >> 8) & 0xffu, where >> 16, pos, pos, (int)seen);
      return m->fail(SPEC_ERR_TIMEOUT, msg);
    }
    return m->fail(SPEC_ERR_INVALID, "a kernel rejected an index (token id out of range?)");
  }
  return SPEC_OK;
}

void fill_step_causal(spec_model* m, const uint32_t* toks, int M, int P) {
  StepDev* st = m->step_host;
  for (int i = 0; i < M; ++i) {
    st->tokens[i] = (int)toks[i];
    st->positions[i] = P + i;
    st->slots[i] = P + i;
    st->anc[i] = (i == 63) ? ~0ull : ((1ull << (i + 1)) - 1ull);
  }
  st->step[0] = P;
  st->step[1] = P + M;
}

// forward_advance_logits (quantized_llama.rs:137-158): forwards `n` tokens
// at cache_len, chunked by kMaxRows; when rows_out != nullptr it receives
// all n logits rows.  On success cache_len += n and the last row is cached.
// True when [p, p + bytes) is page-locked host memory the GPU can copy into
// directly (cudaHostAlloc / cudaHostRegister / a pinned torch tensor).
bool host_pinned(const void* p, size_t bytes) {
  auto one = [](const void* q) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  return one(p) && one(static_cast<const uint8_t*>(p) + bytes - 1);
}

int forward_advance(spec_model* m, const uint32_t* ids, int n, float* rows_out, bool want_logits = true) {
  if (n <= 0) return m->fail(SPEC_ERR_INVALID, "forward_advance with empty tokens");
  if (m->cache_len + n > m->t_max)
    return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded (" + std::to_string(m->cache_len + n) + " > " +
                                         std::to_string(m->t_max) + ")");
  for (int i = 0; i < n; ++i)
    if (ids[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  const int start = m->cache_len;
  const size_t V = (size_t)m->cfg.vocab;
  // Logits rows go straight into a pinned caller buffer; otherwise through
  // the model's pinned staging rows.
  const bool direct = rows_out && host_pinned(rows_out, (size_t)n * V * 4);
  int done = 0;
  while (done < n) {
    const int M = std::min(kMaxRows, n - done);
    fill_step_causal(m, ids + done, M, start + done);
    const bool last_chunk = done + M == n;
    const int flags = (rows_out || (last_chunk && want_logits)) ? F_LOGITS : 0;
    int rc = run_forward(m, M, flags);
    if (rc == SPEC_OK && rows_out) {
      float* dst = direct ? rows_out + (size_t)done * V : m->logits_host;
      const cudaError_t e = cudaMemcpyAsync(dst, m->logits, (size_t)M * V * 4, cudaMemcpyDeviceToHost, m->stream);
      if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "logits rows"));
    }
    if (rc == SPEC_OK) rc = finish(m);
    if (rc != SPEC_OK) {
      m->cache_len = start;  // KV rows beyond cache_len are ignored: state unchanged
      return rc;
    }
    if (rows_out && !direct) memcpy(rows_out + (size_t)done * V, m->logits_host, (size_t)M * V * 4);
    done += M;
  }
  m->cache_len = start + n;
  m->last_valid = want_logits;
  return SPEC_OK;
}

int copy_last_row(spec_model* m, float* out) {
  cudaError_t e = cudaMemcpy(out, m->last_row, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "copy logits"));
  return SPEC_OK;
}

// Tree helpers (crates/speculate/src/tree.rs:38-74, 125-133, 149-158).
int check_tree(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n) {
  if (n <= 0) return m->fail(SPEC_ERR_INVALID, "DraftTree must have at least a root");
  if (n > kMaxRows) return m->fail(SPEC_ERR_UNSUPPORTED, "tree larger than SPEC_MAX_ROWS nodes");
  for (int i = 1; i < n; ++i)
    if (parents[i] < 0 || parents[i] >= i)
      return m->fail(SPEC_ERR_INVALID, "node " + std::to_string(i) + " has parent index " +
                                           std::to_string(parents[i]) + ", which is not strictly smaller");
  for (int i = 0; i < n; ++i)
    if (tokens[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  return SPEC_OK;
}

void fill_step_tree(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, int prefix) {
  StepDev* st = m->step_host;
  for (int i = 0; i < n; ++i) {
    int d = 0;
    unsigned long long anc = 1ull << i;
    for (int cur = i; cur != 0; cur = parents[cur]) {
      ++d;
      anc |= 1ull << parents[cur];
    }
    st->tokens[i] = (int)tokens[i];
    st->positions[i] = prefix + d;
    st->slots[i] = prefix + i;
    st->anc[i] = anc | 1ull;  // the root is everyone's ancestor
  }
  st->step[0] = prefix;
  st->step[1] = prefix + n;
}

int tree_forward(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, int prefix, int flags) {
  if (prefix + n > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  fill_step_tree(m, tokens, parents, n, prefix);
  int rc = run_forward(m, n, flags);
  return rc;
}

}  // namespace

// ===========================================================================
// Model construction
// ===========================================================================
namespace {

int init_device(spec_model* m, const spec_load_opts* opts) {
  m->device = opts ? opts->device : 0;
  m->tp_size = (opts && opts->tp_size > 1) ? opts->tp_size : 1;
  m->tp_rank = m->tp_size > 1 ? opts->tp_rank : 0;
  if (m->tp_rank < 0 || m->tp_rank >= m->tp_size) return m->fail(SPEC_ERR_INVALID, "tp_rank outside [0, tp_size)");
  m->use_graphs = opts ? (opts->use_graphs != 0) : true;
  if (getenv("SPEC_B200_NO_GRAPHS")) m->use_graphs = false;
  if (getenv("SPEC_B200_NO_PDL")) m->use_pdl = false;
  if (getenv("SPEC_B200_FUSED_ATTN")) m->fused_attn = true;
  if (getenv("SPEC_B200_NO_ATTN_TRIGGER")) m->attn_trigger = false;
  if (getenv("SPEC_B200_ATTN_KERNELS_NO_PDL")) m->attn_kernels_pdl = false;
  if (getenv("SPEC_B200_NO_COOP")) m->coop = false;
  if (getenv("SPEC_B200_NO_ROTATE")) m->rotate = false;
  if (getenv("SPEC_B200_NO_EARLY_TRIGGER")) m->early_trigger = false;
  if (const char* env = getenv("SPEC_B200_L2_AHEAD")) m->l2_ahead = atoi(env);
  cudaError_t e = cudaSetDevice(m->device);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "cudaSetDevice"));
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, m->device);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "device properties"));
  if (prop.major < 10) return m->fail(SPEC_ERR_UNSUPPORTED, std::string("needs an sm_100 GPU, found ") + prop.name);
  m->num_sms = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "stream"));
  return SPEC_OK;
}

int upload_vec(spec_model* m, float** dst, const float* src, int n) {
  cudaError_t e = m->dalloc(dst, (size_t)n * 4);
  if (e == cudaSuccess) e = m->upload(*dst, src, (size_t)n * 4);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "upload vector"));
  return SPEC_OK;
}

int finalize_model(spec_model* m, const spec_load_opts* opts, int ctx_len) {
  m->fmt_set = fwd_fmt_set_for(m->fmt_bits);
  if (!m->fmt_set) return m->fail(SPEC_ERR_UNSUPPORTED, "model mixes weight formats no forward kernel covers");
  int want = opts && opts->max_ctx > 0 ? opts->max_ctx : std::min(ctx_len > 0 ? ctx_len : 4096, 4096);
  m->t_max = want;
  int rc = alloc_runtime(m);
  if (rc == SPEC_OK) rc = build_rope(m);
  if (rc == SPEC_OK) {
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "init"));
  }
  return rc;
}

size_t raw_row_bytes(int fmt, int K) { return (size_t)(K / fmt_block_elems(fmt)) * fmt_block_bytes(fmt); }

// Rows [row0, row0 + rows) of a part (a view, no copy).
Part part_rows(const Part& p, int K, int row0, int rows) {
  Part q = p;
  q.src = p.src + (size_t)row0 * raw_row_bytes(p.fmt, K);
  q.rows = rows;
  return q;
}

// Columns [k0, k0 + kn) of every row of a part, gathered into a device buffer
// (whole GGUF blocks; k0 and kn must be multiples of the block width).
int part_cols(spec_model* m, std::vector<void*>& temps, const Part& p, int K, int k0, int kn, Part& out) {
  const int be = fmt_block_elems(p.fmt);
  if (be == 0 || k0 % be || kn % be) return m->fail(SPEC_ERR_UNSUPPORTED, "tensor-parallel column split inside a block");
  const size_t full = raw_row_bytes(p.fmt, K), width = raw_row_bytes(p.fmt, kn), off = raw_row_bytes(p.fmt, k0);
  void* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, width * p.rows);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "shard staging"));
  temps.push_back(buf);
  e = cudaMemcpy2DAsync(buf, width, p.src + off, full, width, p.rows,
                        p.on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "shard copy"));
  out = p;
  out.src = static_cast<const uint8_t*>(buf);
  out.on_device = true;
  return SPEC_OK;
}

// Checks that the model splits into tp_size tensor-parallel shards: whole q
// and kv heads per rank, FFN slices of whole 128-row groups, and column
// splits on tile boundaries.
int check_tp_shape(spec_model* m, int nq, int nkv, int hd, int F, int n_layers) {
  const int N = m->tp_size;
  if (N == 1) return SPEC_OK;
  if (n_layers > kTpMaxLayers) return m->fail(SPEC_ERR_UNSUPPORTED, "too many layers for tensor parallelism");
  if (N > kTpMaxRanks) return m->fail(SPEC_ERR_UNSUPPORTED, "more than 8 tensor-parallel ranks");
  if (nkv % N)
    return m->fail(SPEC_ERR_UNSUPPORTED,
                   "tp_size does not divide the KV heads (KV-head replication across ranks is not built)");
  if (nq % N || F % N || (F / N) % kGroupRows || ((nq / N) * hd) % kGroupRows || ((nkv / N) * hd) % kGroupRows)
    return m->fail(SPEC_ERR_UNSUPPORTED, "model does not split into tp_size tensor-parallel shards");
  return SPEC_OK;
}

// Vocabulary-parallel LM head: rank r keeps 128-row groups
// [r G / T, (r + 1) G / T) of the head's G groups (V rows of K columns in
// GGUF blocks); the other ranks compute the rest and every rank receives all
// rows (EPI_STORE with out_peers).  Records the rank's first row.  Every rank
// needs at least one group.
int shard_lm(spec_model* m, Part& p, int V, int K) {
  m->lm_groups_total = V / kGroupRows;
  m->lm_row0 = 0;
  if (m->tp_size <= 1) return SPEC_OK;
  const int G = m->lm_groups_total, T = m->tp_size, r = m->tp_rank;
  if (G < T) return m->fail(SPEC_ERR_UNSUPPORTED, "vocabulary has fewer 128-row groups than tensor-parallel ranks");
  const int g0 = (int)((long long)r * G / T), g1 = (int)((long long)(r + 1) * G / T);
  const size_t row_bytes = (size_t)(K / fmt_block_elems(p.fmt)) * fmt_block_bytes(p.fmt);
  p.src += (size_t)g0 * kGroupRows * row_bytes;
  p.rows = (g1 - g0) * kGroupRows;
  m->lm_row0 = g0 * kGroupRows;
  return SPEC_OK;
}

// The tensor-parallel shard of one layer for this rank: q/k/v rows of the
// rank's heads and gate/up rows of its FFN slice (column-parallel), the
// o-projection's columns of its heads and the down projection's columns of
// its FFN slice (row-parallel; their outputs are summed across ranks).
// nq, nkv and F are the whole model's.
int shard_layer(spec_model* m, std::vector<void*>& temps, int nq, int nkv, int hd, int H, int F, Part& q, Part& k,
                Part& v, Part& o, Part& g, Part& u, Part& d) {
  const int N = m->tp_size, r = m->tp_rank;
  if (N == 1) return SPEC_OK;
  const int nql = nq / N, nkvl = nkv / N, Fl = F / N;
  q = part_rows(q, H, r * nql * hd, nql * hd);
  k = part_rows(k, H, r * nkvl * hd, nkvl * hd);
  v = part_rows(v, H, r * nkvl * hd, nkvl * hd);
  g = part_rows(g, H, r * Fl, Fl);
  u = part_rows(u, H, r * Fl, Fl);
  // Row-parallel K slices, widened to whole 256-column superblocks (every
  // layer gets the same windows, so the operand layout is per model).
  auto window = [](int K, int k0, int kn, int& lo, int& width, int& off) {
    lo = k0 / 256 * 256;
    const int hi = std::min(K, (k0 + kn + 255) / 256 * 256);
    width = hi - lo;
    off = k0 - lo;
  };
  int o_lo, d_lo;
  window(nq * hd, r * nql * hd, nql * hd, o_lo, m->o_kwin, m->o_koff);
  window(F, r * Fl, Fl, d_lo, m->d_kwin, m->d_koff);
  Part o2, d2;
  int rc = part_cols(m, temps, o, nq * hd, o_lo, m->o_kwin, o2);
  if (rc == SPEC_OK) rc = part_cols(m, temps, d, F, d_lo, m->d_kwin, d2);
  if (rc != SPEC_OK) return rc;
  o = o2;
  d = d2;
  return SPEC_OK;
}

// This rank's slice [q heads | k heads | v heads] of a full q/k/v bias.
std::vector<float> shard_qkv_bias(const spec_model* m, const std::vector<float>& full, int nq, int nkv, int hd) {
  const int N = m->tp_size, r = m->tp_rank;
  if (N == 1) return full;
  const int nql = nq / N, nkvl = nkv / N;
  std::vector<float> out;
  out.insert(out.end(), full.begin() + (size_t)r * nql * hd, full.begin() + (size_t)(r + 1) * nql * hd);
  const size_t kb = (size_t)nq * hd, vb = kb + (size_t)nkv * hd;
  out.insert(out.end(), full.begin() + kb + (size_t)r * nkvl * hd, full.begin() + kb + (size_t)(r + 1) * nkvl * hd);
  out.insert(out.end(), full.begin() + vb + (size_t)r * nkvl * hd, full.begin() + vb + (size_t)(r + 1) * nkvl * hd);
  return out;
}

// After the shards are built, the model's head and FFN counts are this
// rank's (hidden size, vocabulary and head size are whole).
void set_local_dims(spec_model* m) {
  ModelCfg& c = m->cfg;
  c.n_heads /= m->tp_size;
  c.n_kv /= m->tp_size;
  c.ffn /= m->tp_size;
}

int load_from_gguf(spec_model* m, const char* path, const spec_load_opts* opts) {
  GgufFile f;
  std::string err = f.open(path);
  if (!err.empty()) return m->fail(SPEC_ERR_IO, err);
  std::string arch;
  if (!f.get_str("general.architecture", arch)) return m->fail(SPEC_ERR_IO, "missing general.architecture");
  ModelCfg& c = m->cfg;
  if (arch == "llama") c.arch = 0;
  else if (arch == "qwen2") c.arch = 1;
  else return m->fail(SPEC_ERR_UNSUPPORTED, "unsupported architecture " + arch);
  auto need_u32 = [&](const std::string& k, int& out) -> bool {
    uint32_t v;
    if (!f.get_u32(arch + "." + k, v)) {
      m->fail(SPEC_ERR_IO, "cannot find " + arch + "." + k + " in GGUF metadata");
      return false;
    }
    out = (int)v;
    return true;
  };
  if (!need_u32("attention.head_count", c.n_heads) || !need_u32("attention.head_count_kv", c.n_kv) ||
      !need_u32("embedding_length", c.hidden) || !need_u32("context_length", c.ctx_len) ||
      !need_u32("block_count", c.n_layers))
    return SPEC_ERR_IO;
  if (!f.get_f32(arch + ".attention.layer_norm_rms_epsilon", c.eps))
    return m->fail(SPEC_ERR_IO, "cannot find " + arch + ".attention.layer_norm_rms_epsilon in GGUF metadata");
  if (!f.get_f32(arch + ".rope.freq_base", c.rope_theta)) c.rope_theta = 10000.f;
  c.head_dim = c.hidden / c.n_heads;
  c.has_bias = c.arch == 1;
  c.rope_interleaved = c.arch == 0;
  std::string style;
  if (f.get_str("speculate_b200.rope_style", style) && style == "half") c.rope_interleaved = false;
  std::string rs;
  if (f.get_str(arch + ".rope.scaling.type", rs) && rs == "llama3") {
    c.rope_scaled = true;
    f.get_f32(arch + ".rope.scaling.factor", c.rs_factor);
    f.get_f32(arch + ".rope.scaling.low_freq_factor", c.rs_low);
    f.get_f32(arch + ".rope.scaling.high_freq_factor", c.rs_high);
    uint32_t o;
    if (f.get_u32(arch + ".rope.scaling.original_context_length", o)) c.rs_orig = (int)o;
  }
  const GgufValue* toks = f.get("tokenizer.ggml.tokens");
  const GgufTensor* te = f.tensor("token_embd.weight");
  if (!te || te->dims.size() != 2) return m->fail(SPEC_ERR_IO, "missing token_embd.weight");
  c.vocab = toks ? (int)toks->arr_len : (int)te->dims[1];
  if ((int)te->dims[1] < c.vocab) return m->fail(SPEC_ERR_IO, "token_embd has fewer rows than the vocabulary");
  const GgufTensor* g0 = f.tensor("blk.0.ffn_gate.weight");
  if (!g0) return m->fail(SPEC_ERR_IO, "missing blk.0.ffn_gate.weight");
  c.ffn = (int)g0->dims[1];
  c.bf16 = te->type == WF_BF16 || g0->type == WF_BF16;
  c.rope_tables_bf16 = c.bf16 && c.arch == 0;
  if (c.hidden % kGroupRows || c.ffn % kGroupRows || (c.head_dim != 64 && c.head_dim != 128) ||
      c.n_heads % c.n_kv || c.hidden / kGroupRows > kMaxSsGroups)
    return m->fail(SPEC_ERR_UNSUPPORTED, "unsupported model shape");
  if (int rc0 = check_tp_shape(m, c.n_heads, c.n_kv, c.head_dim, c.ffn, c.n_layers)) return rc0;

  auto part_of = [&](const std::string& name, int K, Part& p) -> bool {
    const GgufTensor* t = f.tensor(name);
    if (!t) {
      m->fail(SPEC_ERR_IO, "cannot find tensor " + name);
      return false;
    }
    if (t->dims.size() != 2 || (int)t->dims[0] != K) {
      m->fail(SPEC_ERR_IO, "tensor " + name + " has an unexpected shape");
      return false;
    }
    p.src = f.data(*t);
    p.on_device = false;
    p.fmt = t->type;
    p.rows = (int)t->dims[1];
    return true;
  };
  auto vec_of = [&](const std::string& name, int n, float** dst) -> int {
    const GgufTensor* t = f.tensor(name);
    if (!t) return m->fail(SPEC_ERR_IO, "cannot find tensor " + name);
    uint64_t cnt = 1;
    for (auto d : t->dims) cnt *= d;
    if ((int)cnt != n) return m->fail(SPEC_ERR_IO, "tensor " + name + " has an unexpected size");
    std::vector<float> tmp(n);
    const uint8_t* src = f.data(*t);
    if (t->type == WF_F32) {
      memcpy(tmp.data(), src, (size_t)n * 4);
    } else if (t->type == WF_F16 || t->type == WF_BF16) {
      for (int i = 0; i < n; ++i) {
        uint16_t b;
        memcpy(&b, src + 2 * i, 2);
        if (t->type == WF_BF16) {
          uint32_t u = (uint32_t)b << 16;
          memcpy(&tmp[i], &u, 4);
        } else {
          tmp[i] = half_bits_to_float(b);
        }
      }
    } else {
      return m->fail(SPEC_ERR_UNSUPPORTED, "norm/bias tensor " + name + " must be F32/F16/BF16");
    }
    return upload_vec(m, dst, tmp.data(), n);
  };
  const int H = c.hidden, F = c.ffn, hd = c.head_dim;
  m->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    Layer& L = m->layers[l];
    Part q, k, v, o, g, u, d;
    if (!part_of(pre + "attn_q.weight", H, q) || !part_of(pre + "attn_k.weight", H, k) ||
        !part_of(pre + "attn_v.weight", H, v) || !part_of(pre + "attn_output.weight", c.n_heads * hd, o) ||
        !part_of(pre + "ffn_gate.weight", H, g) || !part_of(pre + "ffn_up.weight", H, u) ||
        !part_of(pre + "ffn_down.weight", F, d))
      return SPEC_ERR_IO;
    if (q.rows != c.n_heads * hd || k.rows != c.n_kv * hd || v.rows != c.n_kv * hd || o.rows != H ||
        g.rows != F || u.rows != F || d.rows != H)
      return m->fail(SPEC_ERR_IO, "layer " + std::to_string(l) + " has inconsistent shapes");
    std::vector<void*> temps;
    m->o_kwin = c.n_heads * hd;  // shard_layer narrows them under tensor parallelism
    m->d_kwin = F;
    int rc = shard_layer(m, temps, c.n_heads, c.n_kv, hd, H, F, q, k, v, o, g, u, d);
    if (rc == SPEC_OK) rc = build_mat(m, {q, k, v}, H, false, L.qkv);
    if (rc == SPEC_OK) rc = build_mat(m, {o}, m->o_kwin, false, L.o);
    if (rc == SPEC_OK) rc = build_mat(m, {g, u}, H, true, L.gu);
    if (rc == SPEC_OK) rc = build_mat(m, {d}, m->d_kwin, false, L.down);
    cudaStreamSynchronize(m->stream);
    for (void* t : temps) cudaFree(t);
    if (rc == SPEC_OK) rc = vec_of(pre + "attn_norm.weight", H, &L.attn_norm);
    if (rc == SPEC_OK) rc = vec_of(pre + "ffn_norm.weight", H, &L.ffn_norm);
    if (rc == SPEC_OK && c.has_bias) {
      std::vector<float> b((size_t)(c.n_heads + 2 * c.n_kv) * hd);
      float* tmpd = nullptr;
      const char* names[3] = {"attn_q.bias", "attn_k.bias", "attn_v.bias"};
      const int lens[3] = {c.n_heads * hd, c.n_kv * hd, c.n_kv * hd};
      size_t off = 0;
      for (int i = 0; i < 3 && rc == SPEC_OK; ++i) {
        const GgufTensor* t = f.tensor(pre + names[i]);
        if (!t || t->type != WF_F32 || (int)(t->nbytes / 4) != lens[i]) {
          rc = m->fail(SPEC_ERR_IO, "cannot find F32 tensor " + pre + names[i]);
          break;
        }
        memcpy(b.data() + off, f.data(*t), (size_t)lens[i] * 4);
        off += lens[i];
      }
      if (rc == SPEC_OK) {
        std::vector<float> bl = shard_qkv_bias(m, b, c.n_heads, c.n_kv, hd);
        rc = upload_vec(m, &tmpd, bl.data(), (int)bl.size());
      }
      L.bqkv = tmpd;
    }
    if (rc != SPEC_OK) return rc;
  }
  int rc = vec_of("output_norm.weight", H, &m->out_norm);
  if (rc != SPEC_OK) return rc;
  // Embedding table stays in its GGUF layout for the gather.
  m->embed_fmt = te->type;
  if (fmt_block_elems(te->type) == 0 || H % fmt_block_elems(te->type))
    return m->fail(SPEC_ERR_UNSUPPORTED, "unsupported token_embd format");
  {
    cudaError_t e = m->dalloc(&m->embed_raw, te->nbytes);
    if (e == cudaSuccess) e = m->upload(m->embed_raw, f.data(*te), te->nbytes);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "embedding upload"));
  }
  Part outp;
  const GgufTensor* ot = f.tensor("output.weight");
  if (ot) {
    if (!part_of("output.weight", H, outp)) return SPEC_ERR_IO;
  } else {  // tied weights (quantized_llama_local.rs:249-252)
    if (!part_of("token_embd.weight", H, outp)) return SPEC_ERR_IO;
  }
  if (outp.rows < c.vocab) return m->fail(SPEC_ERR_IO, "output.weight has fewer rows than the vocabulary");
  if (c.vocab % kGroupRows) return m->fail(SPEC_ERR_UNSUPPORTED, "vocabulary not a multiple of 128");
  outp.rows = c.vocab;
  rc = shard_lm(m, outp, c.vocab, H);
  if (rc == SPEC_OK) rc = build_mat(m, {outp}, H, false, m->lm);
  if (rc != SPEC_OK) return rc;
  set_local_dims(m);
  return finalize_model(m, opts, c.ctx_len);
}

}  // namespace

// ===========================================================================
// Synthetic models
// ===========================================================================
namespace {

int mix_type(int mix, bool is_output, bool is_v_or_down, int layer, int K) {
  if (mix == 3) return WF_BF16;
  if (mix == 2) return WF_Q8_0;
  int base;
  if (is_output) base = WF_Q6_K;
  else if (mix == 0) base = (layer >= 0 && layer % 2 == 0 && is_v_or_down) ? WF_Q6_K : WF_Q4_K;
  else base = WF_Q5_K;
  if (K % 256) return WF_Q8_0;
  return base;
}

uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Raw GGUF blocks for one seeded tensor, generated on the device.
int synth_part(spec_model* m, std::vector<void*>& temps, int fmt, int rows, int K, uint64_t seed, Part& p,
               float sigma = 0.02f) {
  const size_t bytes = (size_t)rows * (K / fmt_block_elems(fmt)) * fmt_block_bytes(fmt);
  void* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, bytes);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "synthetic staging"));
  temps.push_back(buf);
  e = launch_synth_quant(static_cast<uint8_t*>(buf), fmt, rows, K, seed, sigma, 0, m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "synthetic weights"));
  p.src = static_cast<const uint8_t*>(buf);
  p.on_device = true;
  p.fmt = fmt;
  p.rows = rows;
  return SPEC_OK;
}

int synth_vec(spec_model* m, float** dst, int n, uint64_t seed, float base) {
  cudaError_t e = m->dalloc(dst, (size_t)n * 4);
  if (e == cudaSuccess) e = launch_synth_vec(*dst, n, seed, base, 0.02f, m->stream);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "synthetic vector"));
  return SPEC_OK;
}

int create_synthetic(spec_model* m, const spec_model_desc* d, uint64_t seed, const spec_load_opts* opts) {
  ModelCfg& c = m->cfg;
  c.arch = d->arch;
  c.n_layers = d->n_layers;
  c.hidden = d->hidden;
  c.n_heads = d->n_heads;
  c.n_kv = d->n_kv_heads;
  c.ffn = d->ffn;
  c.vocab = d->vocab;
  c.rope_theta = d->rope_theta;
  c.eps = d->eps;
  c.head_dim = c.hidden / c.n_heads;
  c.has_bias = c.arch == 1;
  c.bf16 = d->quant_mix == 3;
  c.rope_interleaved = c.arch == 0 && !d->rope_half;
  c.rope_tables_bf16 = c.bf16 && c.arch == 0;
  c.ctx_len = 131072;
  if (c.bf16 && c.arch == 0) {  // Llama-3.1 frequency scaling for the BF16 checkpoint shape
    c.rope_scaled = true;
  }
  if (c.n_layers <= 0 || c.hidden % kGroupRows || c.ffn % kGroupRows || c.vocab % kGroupRows ||
      c.hidden / kGroupRows > kMaxSsGroups ||
      (c.head_dim != 64 && c.head_dim != 128) || c.n_heads % c.n_kv)
    return m->fail(SPEC_ERR_UNSUPPORTED, "unsupported synthetic model shape");
  if (int rc0 = check_tp_shape(m, c.n_heads, c.n_kv, c.head_dim, c.ffn, c.n_layers)) return rc0;
  const int H = c.hidden, F = c.ffn, hd = c.head_dim;
  uint64_t tid = 0;
  auto tseed = [&]() { return spec_synthetic_seed(seed, ++tid); };  // tensor numbering: spec_b200.h
  // Output norm, embedding and head first, so a shallower model with the
  // same seed shares them.
  {
    const int rc0 = synth_vec(m, &m->out_norm, H, tseed(), 1.f);
    if (rc0 != SPEC_OK) return rc0;
  }
  {
    std::vector<void*> temps;
    Part ep, op;
    m->embed_fmt = mix_type(d->quant_mix, false, false, -1, H);
    int rc = synth_part(m, temps, m->embed_fmt, c.vocab, H, tseed(), ep);
    if (rc == SPEC_OK) {
      const size_t bytes = (size_t)c.vocab * (H / fmt_block_elems(m->embed_fmt)) * fmt_block_bytes(m->embed_fmt);
      cudaError_t e = m->dalloc(&m->embed_raw, bytes);
      if (e == cudaSuccess) e = cudaMemcpyAsync(m->embed_raw, ep.src, bytes, cudaMemcpyDeviceToDevice, m->stream);
      if (e != cudaSuccess) rc = m->fail(SPEC_ERR_OOM, cuda_msg(e, "embedding"));
    }
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(d->quant_mix, true, false, -1, H), c.vocab, H, tseed(), op);
    if (rc == SPEC_OK) {
      rc = shard_lm(m, op, c.vocab, H);
      if (rc == SPEC_OK) rc = build_mat(m, {op}, H, false, m->lm);
    }
    cudaStreamSynchronize(m->stream);
    for (void* t : temps) cudaFree(t);
    if (rc != SPEC_OK) return rc;
  }
  const bool damp_on = d->damp_from_layer > 0;
  const float damp_sigma = 0.02f * (float)d->damp_e4 / 10000.f;
  m->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    Layer& L = m->layers[l];
    std::vector<void*> temps;
    Part q, k, v, o, g, u, dn;
    const int mix = d->quant_mix;
    int rc = synth_part(m, temps, mix_type(mix, false, false, l, H), c.n_heads * hd, H, tseed(), q);
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(mix, false, false, l, H), c.n_kv * hd, H, tseed(), k);
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(mix, false, true, l, H), c.n_kv * hd, H, tseed(), v);
    const float sig_od = (damp_on && l >= d->damp_from_layer) ? damp_sigma : 0.02f;
    if (rc == SPEC_OK)
      rc = synth_part(m, temps, mix_type(mix, false, false, l, c.n_heads * hd), H, c.n_heads * hd, tseed(), o, sig_od);
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(mix, false, false, l, H), F, H, tseed(), g);
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(mix, false, false, l, H), F, H, tseed(), u);
    if (rc == SPEC_OK) rc = synth_part(m, temps, mix_type(mix, false, true, l, F), H, F, tseed(), dn, sig_od);
    m->o_kwin = c.n_heads * hd;  // shard_layer narrows them under tensor parallelism
    m->d_kwin = F;
    if (rc == SPEC_OK) rc = shard_layer(m, temps, c.n_heads, c.n_kv, hd, H, F, q, k, v, o, g, u, dn);
    if (rc == SPEC_OK) rc = build_mat(m, {q, k, v}, H, false, L.qkv);
    if (rc == SPEC_OK) rc = build_mat(m, {o}, m->o_kwin, false, L.o);
    if (rc == SPEC_OK) rc = build_mat(m, {g, u}, H, true, L.gu);
    if (rc == SPEC_OK) rc = build_mat(m, {dn}, m->d_kwin, false, L.down);
    if (rc == SPEC_OK) rc = synth_vec(m, &L.attn_norm, H, tseed(), 1.f);
    if (rc == SPEC_OK) rc = synth_vec(m, &L.ffn_norm, H, tseed(), 1.f);
    if (rc == SPEC_OK && c.has_bias) {
      const int nb = (c.n_heads + 2 * c.n_kv) * hd;
      float* full = nullptr;
      rc = synth_vec(m, &full, nb, tseed(), 0.f);
      if (rc == SPEC_OK && m->tp_size > 1) {
        std::vector<float> h(nb);
        cudaError_t e = cudaMemcpyAsync(h.data(), full, (size_t)nb * 4, cudaMemcpyDeviceToHost, m->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
        if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "bias shard"));
        std::vector<float> b = shard_qkv_bias(m, h, c.n_heads, c.n_kv, hd);
        if (rc == SPEC_OK) rc = upload_vec(m, &L.bqkv, b.data(), (int)b.size());
      } else {
        L.bqkv = full;
      }
    }
    cudaStreamSynchronize(m->stream);
    for (void* t : temps) cudaFree(t);
    if (rc != SPEC_OK) return rc;
  }
  set_local_dims(m);
  return finalize_model(m, opts, c.ctx_len);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int spec_load_gguf(const char* path, const spec_load_opts* opts, spec_model** out) {
  if (!out || !path) {
    g_load_error = "null argument";
    return SPEC_ERR_INVALID;
  }
  *out = nullptr;
  std::unique_ptr<spec_model> m(new (std::nothrow) spec_model());
  if (!m) return SPEC_ERR_OOM;
  DeviceGuard dg_(opts ? opts->device : 0);
  int rc = init_device(m.get(), opts);
  if (rc == SPEC_OK) rc = load_from_gguf(m.get(), path, opts);
  if (rc != SPEC_OK) {
    g_load_error = m->err;
    return rc;
  }
  *out = m.release();
  return SPEC_OK;
}

int spec_create_synthetic(const spec_model_desc* desc, uint64_t seed, const spec_load_opts* opts,
                          spec_model** out) {
  if (!out || !desc) {
    g_load_error = "null argument";
    return SPEC_ERR_INVALID;
  }
  *out = nullptr;
  std::unique_ptr<spec_model> m(new (std::nothrow) spec_model());
  if (!m) return SPEC_ERR_OOM;
  DeviceGuard dg_(opts ? opts->device : 0);
  int rc = init_device(m.get(), opts);
  if (rc == SPEC_OK) rc = create_synthetic(m.get(), desc, seed, opts);
  if (rc != SPEC_OK) {
    g_load_error = m->err;
    return rc;
  }
  *out = m.release();
  return SPEC_OK;
}

void spec_free(spec_model* m) { delete m; }

uint64_t spec_synthetic_seed(uint64_t model_seed, uint64_t index) {
  return mix64(model_seed * 0x100000001B3ull + index);
}

int spec_synthetic_tensor(int device, int ggml_type, int rows, int k_cols, uint64_t seed, float sigma,
                          void* host_out, int64_t out_bytes) {
  const bool known = ggml_type == WF_Q4_K || ggml_type == WF_Q5_K || ggml_type == WF_Q6_K ||
                     ggml_type == WF_Q8_0 || ggml_type == WF_BF16 || ggml_type == WF_F16 || ggml_type == WF_F32;
  if (!host_out || rows <= 0 || k_cols <= 0 || !known || k_cols % fmt_block_elems(ggml_type)) {
    g_load_error = "spec_synthetic_tensor: null output, bad shape or unsupported type";
    return SPEC_ERR_INVALID;
  }
  const size_t bytes = (size_t)rows * (size_t)(k_cols / fmt_block_elems(ggml_type)) * fmt_block_bytes(ggml_type);
  if (out_bytes < (int64_t)bytes) {
    g_load_error = "spec_synthetic_tensor: output buffer too small";
    return SPEC_ERR_INVALID;
  }
  DeviceGuard dg_(device);
  void* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, bytes);
  if (e == cudaSuccess) e = launch_synth_quant(static_cast<uint8_t*>(buf), ggml_type, rows, k_cols, seed, sigma, 0, 0);
  if (e == cudaSuccess) e = cudaMemcpy(host_out, buf, bytes, cudaMemcpyDeviceToHost);
  if (buf) cudaFree(buf);
  if (e != cudaSuccess) {
    g_load_error = cuda_msg(e, "spec_synthetic_tensor");
    return SPEC_ERR_CUDA;
  }
  return SPEC_OK;
}

int spec_synthetic_vector(int device, int n, uint64_t seed, float base, float sigma, float* host_out) {
  if (!host_out || n <= 0) {
    g_load_error = "spec_synthetic_vector: null output or n <= 0";
    return SPEC_ERR_INVALID;
  }
  DeviceGuard dg_(device);
  float* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, (size_t)n * 4);
  if (e == cudaSuccess) e = launch_synth_vec(buf, n, seed, base, sigma, 0);
  if (e == cudaSuccess) e = cudaMemcpy(host_out, buf, (size_t)n * 4, cudaMemcpyDeviceToHost);
  if (buf) cudaFree(buf);
  if (e != cudaSuccess) {
    g_load_error = cuda_msg(e, "spec_synthetic_vector");
    return SPEC_ERR_CUDA;
  }
  return SPEC_OK;
}

int spec_tp_handle(spec_model* m, void* out, int cap) {
  if (!m || !out) return -SPEC_ERR_INVALID;
  if (m->tp_size <= 1 || !m->tp_buf) return -m->fail(SPEC_ERR_INVALID, "not a tensor-parallel handle");
  if (cap < (int)sizeof(cudaIpcMemHandle_t)) return -m->fail(SPEC_ERR_INVALID, "handle buffer too small");
  DeviceGuard dg_(m->device);
  // The zeroed counters must be in place before any peer can write to them.
  cudaError_t e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return -m->fail(SPEC_ERR_CUDA, cuda_msg(e, "stream"));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, m->tp_buf);
  if (e != cudaSuccess) return -m->fail(SPEC_ERR_CUDA, cuda_msg(e, "cudaIpcGetMemHandle"));
  memcpy(out, &h, sizeof h);
  return (int)sizeof h;
}

int spec_tp_connect(spec_model* m, const void* handles, int n) {
  if (!m || !handles) return SPEC_ERR_INVALID;
  if (m->tp_size <= 1 || n != m->tp_size) return m->fail(SPEC_ERR_INVALID, "handle count differs from tp_size");
  if (m->tp_connected) return m->fail(SPEC_ERR_INVALID, "already connected");
  DeviceGuard dg_(m->device);
  std::vector<uint8_t*> base(n);
  for (int r = 0; r < n; ++r) {
    if (r == m->tp_rank) {
      base[r] = m->tp_buf;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof h, sizeof h);
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "cudaIpcOpenMemHandle"));
    m->tp_peer_bases.push_back(ptr);
    base[r] = static_cast<uint8_t*>(ptr);
  }
  std::vector<void*> ptrs((size_t)2 * n);
  for (int set = 0; set < 2; ++set)
    for (int r = 0; r < n; ++r) ptrs[(size_t)set * n + r] = base[r] + set * m->tp_set_bytes;
  std::vector<float*> outs(n);
  std::vector<unsigned long long*> ctrs(n);
  for (int r = 0; r < n; ++r) {
    outs[r] = reinterpret_cast<float*>(base[r] + m->tp_logits_off) + m->lm_row0;
    ctrs[r] = reinterpret_cast<unsigned long long*>(base[r] + m->tp_counter_off);
  }
  cudaError_t e = m->upload(m->tp_ptrs_dev, ptrs.data(), ptrs.size() * sizeof(void*));
  if (e == cudaSuccess) e = m->upload(m->tp_out_peers_dev, outs.data(), outs.size() * sizeof(float*));
  if (e == cudaSuccess) e = m->upload(m->tp_out_counters_dev, ctrs.data(), ctrs.size() * sizeof(void*));
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "peer pointer table"));
  m->tp_connected = true;
  return SPEC_OK;
}

int spec_tp_size(const spec_model* m) { return m ? m->tp_size : 0; }

const char* spec_last_error(const spec_model* m) { return m ? m->err.c_str() : g_load_error.c_str(); }

int spec_vocab_size(const spec_model* m) { return m ? m->cfg.vocab : 0; }
int spec_hidden_size(const spec_model* m) { return m ? m->cfg.hidden : 0; }
int spec_num_layers(const spec_model* m) { return m ? m->cfg.n_layers : 0; }
int spec_history_len(const spec_model* m) { return m ? (int)m->history.size() : 0; }
int spec_history(const spec_model* m, uint32_t* out, int cap) {
  if (!m) return 0;
  const int n = (int)m->history.size();
  if (out && cap > 0) memcpy(out, m->history.data(), (size_t)std::min(cap, n) * 4);
  return n;
}
// The logical KV length: a pending last token (lazy observe) counts.
int spec_kv_len(const spec_model* m) {
  if (!m) return 0;
  return m->cache_len + (m->cache_len == (int)m->history.size() - 1 ? 1 : 0);
}
int spec_max_ctx(const spec_model* m) { return m ? m->t_max : 0; }

int spec_reset(spec_model* m) {
  if (!m) return SPEC_ERR_INVALID;
  m->history.clear();
  m->cache_len = 0;
  m->last_valid = false;
  return SPEC_OK;
}

// Lazy observe: the KV rows of every new token but the last are computed
// now; the last token stays pending (cache_len == history - 1) and its row is
// computed by the next call that needs it -- next_logits, batched_logits, a
// tree or verify forward -- which recompute the last committed token anyway
// (quantized_llama.rs:561-569 truncates and replays it).  So the M=1 forward
// that vanilla SD's observe runs after each round (vanilla.rs:358-360) is
// folded into the next verify.  Rows are bit-identical either way: every
// row's arithmetic is independent of the rows batched with it.
int spec_observe(spec_model* m, const uint32_t* ids, int n) {
  if (!m || (n > 0 && !ids) || n < 0) return SPEC_ERR_INVALID;
  if (n == 0) return SPEC_OK;
  DeviceGuard dg_(m->device);
  for (int i = 0; i < n; ++i)
    if (ids[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  const int size = (int)m->history.size();
  if (size + n > m->t_max)
    return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded (" + std::to_string(size + n) + " > " +
                                         std::to_string(m->t_max) + ")");
  std::vector<uint32_t> todo;
  if (size > 0 && m->cache_len == size - 1) todo.push_back(m->history.back());
  todo.insert(todo.end(), ids, ids + n - 1);
  if (!todo.empty()) {
    const int rc = forward_advance(m, todo.data(), (int)todo.size(), nullptr, false);
    if (rc != SPEC_OK) return rc;
  }
  m->history.insert(m->history.end(), ids, ids + n);
  m->last_valid = false;
  return SPEC_OK;
}

int spec_next_logits(spec_model* m, float* out) {
  if (!m || !out) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "next_logits called with empty history");
  if (m->last_valid) return copy_last_row(m, out);
  const uint32_t last = m->history.back();
  const int saved = m->cache_len;
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  m->cache_len = target;
  int rc = forward_advance(m, &last, 1, nullptr);
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    return rc;
  }
  return copy_last_row(m, out);
}

int spec_batched_logits(spec_model* m, const uint32_t* drafts, int k, float* out) {
  if (!m || !out || k < 0 || (k > 0 && !drafts)) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (k == 0) return spec_next_logits(m, out);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "batched_logits with empty history");
  std::vector<uint32_t> combined(k + 1);
  combined[0] = m->history.back();
  memcpy(combined.data() + 1, drafts, (size_t)k * 4);
  const int saved = m->cache_len;
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  const bool saved_valid = m->last_valid;
  m->cache_len = target;
  int rc = forward_advance(m, combined.data(), k + 1, out);
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    m->last_valid = saved_valid;
    return rc;
  }
  m->history.insert(m->history.end(), drafts, drafts + k);
  return SPEC_OK;
}

int spec_rollback_to(spec_model* m, int len) {
  if (!m || len < 0) return SPEC_ERR_INVALID;
  if (len > (int)m->history.size())
    return m->fail(SPEC_ERR_CACHE_ROLLBACK, "rollback target " + std::to_string(len) + " > history length " +
                                                std::to_string(m->history.size()));
  const int logical = spec_kv_len(m);
  if (len > logical)
    return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate_kv_cache_to(" + std::to_string(len) + ") exceeds " +
                                                std::to_string(logical));
  const bool keep_valid = m->last_valid && len == (int)m->history.size() && m->cache_len == len;
  m->history.resize(len);
  m->last_valid = keep_valid;
  // A pending last token (cache_len == len - 1) stays pending.
  m->cache_len = std::min(m->cache_len, len);
  return SPEC_OK;
}

// A tree of more than kMaxRows nodes, cut into forwards of at most kMaxRows
// rows.  Nodes are taken in index order; each joins the current chunk with
// every ancestor it lacks there, or, when they do not fit, starts the next
// chunk with its ancestor chain.  A chunk is closed under ancestors, so it is
// itself a tree rooted at node 0 in which every row attends to exactly its
// own ancestors (and, as in one forward, to the whole prefix); its RoPE
// positions are prefix + depth as before.  A node's logits come from the
// chunk that took it as `primary`; ancestors repeated in later chunks only
// provide keys.
struct TreeChunk {
  std::vector<int> nodes;    // global node indices, ascending
  std::vector<int> primary;  // global nodes whose logits this chunk provides
};

static int plan_tree_chunks(spec_model* m, const int32_t* parents, int n, std::vector<TreeChunk>& chunks) {
  chunks.clear();
  std::vector<char> in(n, 0);
  std::vector<int> chain;
  TreeChunk cur;
  for (int i = 0; i < n; ++i) {
    chain.clear();
    for (int a = i;; a = parents[a]) {
      chain.push_back(a);
      if (a == 0) break;
    }
    if ((int)chain.size() > kMaxRows) return m->fail(SPEC_ERR_UNSUPPORTED, "tree deeper than SPEC_MAX_ROWS - 1");
    int missing = 0;
    for (int a : chain) missing += !in[a];
    if ((int)cur.nodes.size() + missing > kMaxRows) {
      for (int g : cur.nodes) in[g] = 0;
      chunks.push_back(std::move(cur));
      cur = TreeChunk();
    }
    for (int a : chain)
      if (!in[a]) {
        in[a] = 1;
        cur.nodes.push_back(a);
      }
    cur.primary.push_back(i);
  }
  if (!cur.nodes.empty()) chunks.push_back(std::move(cur));
  for (TreeChunk& c : chunks) std::sort(c.nodes.begin(), c.nodes.end());
  return SPEC_OK;
}

// FNV-1a over a tree's size, tokens and parents: identifies the tree whose
// last chunk is in the KV window.
static uint64_t tree_signature(const uint32_t* tokens, const int32_t* parents, int n) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](uint32_t v) {
    for (int b = 0; b < 4; ++b) {
      h ^= (v >> (8 * b)) & 0xffu;
      h *= 1099511628211ull;
    }
  };
  mix((uint32_t)n);
  for (int i = 0; i < n; ++i) {
    mix(tokens[i]);
    mix((uint32_t)(i ? parents[i] : 0));
  }
  return h ? h : 1;
}

static int check_big_tree(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n) {
  for (int i = 1; i < n; ++i)
    if (parents[i] < 0 || parents[i] >= i)
      return m->fail(SPEC_ERR_INVALID, "node " + std::to_string(i) + " has parent index " +
                                           std::to_string(parents[i]) + ", which is not strictly smaller");
  for (int i = 0; i < n; ++i)
    if (tokens[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  return SPEC_OK;
}

// Tokens and local parents of one chunk; local[] maps global -> slot.
static void chunk_arrays(const TreeChunk& c, const uint32_t* tokens, const int32_t* parents, std::vector<int>& local,
                         uint32_t* lt, int32_t* lp) {
  const int cn = (int)c.nodes.size();
  for (int j = 0; j < cn; ++j) local[c.nodes[j]] = j;
  for (int j = 0; j < cn; ++j) {
    const int g = c.nodes[j];
    lt[j] = tokens[g];
    lp[j] = j ? local[parents[g]] : 0;
  }
}

// The forwards of a tree over kMaxRows nodes at `prefix`, one per chunk: the
// primary rows' logits (logits_out, n x V), final hidden rows (hidden_out,
// n x H) and argmaxes (argmax_out, n) go to the host, any of them NULL.  The
// last chunk's KV rows stay in the tree window and are recorded.
// `per_chunk`, when given, runs after each chunk's forward on the model's
// stream with the chunk's rows in m->logits (`local`: global -> row).
using ChunkHook = std::function<int(const TreeChunk&, const std::vector<int>&)>;

static int big_tree_run(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, int prefix,
                        float* logits_out, float* hidden_out, int32_t* argmax_out,
                        const ChunkHook& per_chunk = nullptr) {
  std::vector<TreeChunk> chunks;
  int rc = plan_tree_chunks(m, parents, n, chunks);
  if (rc != SPEC_OK) return rc;
  const size_t V = (size_t)m->cfg.vocab, H = (size_t)m->cfg.hidden;
  const int flags = (logits_out || argmax_out || per_chunk ? F_LOGITS : 0) | (hidden_out ? F_HIDDEN : 0);
  std::vector<int> local(n, -1);
  uint32_t lt[kMaxRows];
  int32_t lp[kMaxRows];
  for (const TreeChunk& c : chunks) {
    const int cn = (int)c.nodes.size();
    chunk_arrays(c, tokens, parents, local, lt, lp);
    rc = tree_forward(m, lt, lp, cn, prefix, flags);
    cudaError_t e = cudaSuccess;
    if (rc == SPEC_OK && logits_out)
      e = cudaMemcpyAsync(m->logits_host, m->logits, (size_t)cn * V * 4, cudaMemcpyDeviceToHost, m->stream);
    if (rc == SPEC_OK && hidden_out && e == cudaSuccess)
      e = cudaMemcpyAsync(m->hidden_host, m->hidden_out, (size_t)cn * H * 4, cudaMemcpyDeviceToHost, m->stream);
    if (rc == SPEC_OK && argmax_out && e == cudaSuccess) {
      e = launch_row_argmax(m->logits, cn, (int)V, m->argmax_dev, nullptr, m->argmax_slots, m->argmax_counters,
                            m->stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->argmax_host, m->argmax_dev, (size_t)cn * 4, cudaMemcpyDeviceToHost, m->stream);
    }
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "tree chunk outputs"));
    if (rc == SPEC_OK && per_chunk) rc = per_chunk(c, local);
    if (rc == SPEC_OK) rc = finish(m);
    if (rc != SPEC_OK) return rc;
    for (int g : c.primary) {
      const int j = local[g];
      if (logits_out) memcpy(logits_out + (size_t)g * V, m->logits_host + (size_t)j * V, V * 4);
      if (hidden_out) memcpy(hidden_out + (size_t)g * H, m->hidden_host + (size_t)j * H, H * 4);
      if (argmax_out) argmax_out[g] = m->argmax_host[j];
    }
  }
  m->tree_window = chunks.back().nodes;
  m->tree_window_sig = tree_signature(tokens, parents, n);
  return SPEC_OK;
}

// spec_tree_logits for trees over kMaxRows nodes: the chunk forwards, then
// the same restore as the single-forward path.
static int big_tree_logits(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float* out) {
  int rc = check_big_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  const uint32_t last = m->history.back();
  if (tokens[0] != last)
    return m->fail(SPEC_ERR_INVALID, "tree root (" + std::to_string(tokens[0]) +
                                         ") must equal last committed token (" + std::to_string(last) + ")");
  const int pre = m->cache_len;
  const int prefix = (int)m->history.size() - 1;
  if (prefix > pre) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  if (prefix + kMaxRows > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  rc = big_tree_run(m, tokens, parents, n, prefix, out, nullptr, nullptr);
  if (rc != SPEC_OK) return rc;
  m->cache_len = prefix;
  rc = forward_advance(m, &last, 1, nullptr);
  if (rc != SPEC_OK) {
    m->cache_len = pre;
    return rc;
  }
  return copy_last_row(m, out);
}

int spec_tree_logits(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float* out) {
  if (!m || !tokens || !parents || !out) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  if (n > kMaxRows) return big_tree_logits(m, tokens, parents, n, out);
  int rc = check_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  const uint32_t last = m->history.back();
  if (tokens[0] != last)
    return m->fail(SPEC_ERR_INVALID, "tree root (" + std::to_string(tokens[0]) +
                                         ") must equal last committed token (" + std::to_string(last) + ")");
  // The root is the last committed token, at position history - 1 (its KV
  // row may still be pending after a lazy observe; the tree forward writes it).
  const int pre = m->cache_len;
  const int prefix = (int)m->history.size() - 1;
  if (prefix > pre) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  rc = tree_forward(m, tokens, parents, n, prefix, F_LOGITS);
  const size_t lbytes = (size_t)n * m->cfg.vocab * 4;
  const bool direct = host_pinned(out, lbytes);  // DMA straight into a pinned caller array
  if (rc == SPEC_OK)
    cudaMemcpyAsync(direct ? out : m->logits_host, m->logits, lbytes, cudaMemcpyDeviceToHost, m->stream);
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) return rc;
  if (!direct) memcpy(out, m->logits_host, lbytes);
  // Restore (quantized_llama.rs:306-323): truncate to prefix and re-forward
  // the root; its logits replace row 0 and become the cached next logits.
  m->cache_len = prefix;
  rc = forward_advance(m, &last, 1, nullptr);
  if (rc != SPEC_OK) {
    m->cache_len = pre;
    return rc;
  }
  return copy_last_row(m, out);
}

// Over kMaxRows nodes: the chunk forwards; the KV window keeps the last
// chunk's rows (cache_len = prefix + its size) and spec_commit_tree_path
// brings the accepted path's chunk back when it is another one.
static int big_tree_keep_kv(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float* logits_out,
                            float* hidden_out, int32_t* argmax_out, const ChunkHook& per_chunk = nullptr) {
  int rc = check_big_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  const uint32_t last = m->history.back();
  if (tokens[0] != last)
    return m->fail(SPEC_ERR_INVALID, "tree root (" + std::to_string(tokens[0]) +
                                         ") must equal last committed token (" + std::to_string(last) + ")");
  const int prefix = (int)m->history.size() - 1;
  if (prefix > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  if (prefix + kMaxRows > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  rc = big_tree_run(m, tokens, parents, n, prefix, logits_out, hidden_out, argmax_out, per_chunk);
  if (rc != SPEC_OK) return rc;
  m->cache_len = prefix + (int)m->tree_window.size();
  return SPEC_OK;
}

int spec_tree_logits_keep_kv(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                             float* logits_out, float* hidden_out) {
  if (!m || !tokens || !parents) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  if (n > kMaxRows) return big_tree_keep_kv(m, tokens, parents, n, logits_out, hidden_out, nullptr);
  int rc = check_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  const uint32_t last = m->history.back();
  if (tokens[0] != last)
    return m->fail(SPEC_ERR_INVALID, "tree root (" + std::to_string(tokens[0]) +
                                         ") must equal last committed token (" + std::to_string(last) + ")");
  // The root is the last committed token, at position history - 1 (its KV
  // row may still be pending after a lazy observe; the tree forward writes it).
  const int pre = m->cache_len;
  const int prefix = (int)m->history.size() - 1;
  if (prefix > pre) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  rc = tree_forward(m, tokens, parents, n, prefix, F_LOGITS | F_HIDDEN);
  const size_t lbytes = (size_t)n * m->cfg.vocab * 4, hbytes = (size_t)n * m->cfg.hidden * 4;
  const bool ldirect = logits_out && host_pinned(logits_out, lbytes);  // DMA into pinned caller arrays
  const bool hdirect = hidden_out && host_pinned(hidden_out, hbytes);
  if (rc == SPEC_OK && logits_out)
    cudaMemcpyAsync(ldirect ? logits_out : m->logits_host, m->logits, lbytes, cudaMemcpyDeviceToHost, m->stream);
  if (rc == SPEC_OK && hidden_out)
    cudaMemcpyAsync(hdirect ? hidden_out : m->hidden_host, m->hidden_out, hbytes, cudaMemcpyDeviceToHost, m->stream);
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) return rc;
  m->cache_len = prefix + n;
  if (logits_out && !ldirect) memcpy(logits_out, m->logits_host, lbytes);
  if (hidden_out && !hdirect) memcpy(hidden_out, m->hidden_host, hbytes);
  return SPEC_OK;
}

int spec_commit_tree_path(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                          const int32_t* accepted, int n_acc) {
  if (!m || !tokens || !parents || !accepted) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "commit_tree_path with empty history");
  const bool big = n > kMaxRows;
  int rc = big ? check_big_tree(m, tokens, parents, n) : check_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  if (n_acc < 1 || accepted[0] != 0) return m->fail(SPEC_ERR_INVALID, "accepted path must start at the root (0)");
  const int prefix = (int)m->history.size() - 1;
  for (int i = 0; i < n_acc; ++i)
    if (accepted[i] < 0 || accepted[i] >= n) return m->fail(SPEC_ERR_INVALID, "accepted index out of range");
  // slot[i]: the tree-window slot holding accepted[i]'s KV row.
  std::vector<int> slot(n_acc);
  if (!big) {
    for (int i = 0; i < n_acc; ++i) {
      if (prefix + accepted[i] >= m->cache_len)
        return m->fail(SPEC_ERR_INVALID, "accepted node is not in the KV cache");
      slot[i] = accepted[i];
    }
  } else {
    // A tree over kMaxRows nodes: the path must be a chain from the root
    // (its nodes are then in one chunk), and that chunk's rows must be in the
    // window, brought back by its forward if the window holds another one.
    for (int i = 1; i < n_acc; ++i)
      if (parents[accepted[i]] != accepted[i - 1])
        return m->fail(SPEC_ERR_UNSUPPORTED, "over SPEC_MAX_ROWS nodes the accepted nodes must form a root path");
    if (m->tree_window_sig == 0 || m->tree_window_sig != tree_signature(tokens, parents, n) ||
        prefix + (int)m->tree_window.size() != m->cache_len)
      return m->fail(SPEC_ERR_INVALID, "accepted node is not in the KV cache");
    std::vector<int> local(n, -1);
    for (size_t j = 0; j < m->tree_window.size(); ++j) local[m->tree_window[j]] = (int)j;
    bool in_window = true;
    for (int i = 0; i < n_acc; ++i) in_window &= local[accepted[i]] >= 0;
    if (!in_window) {
      std::vector<TreeChunk> chunks;
      rc = plan_tree_chunks(m, parents, n, chunks);
      if (rc != SPEC_OK) return rc;
      const int want = accepted[n_acc - 1];
      const TreeChunk* hit = nullptr;
      for (const TreeChunk& c : chunks)
        if (std::find(c.primary.begin(), c.primary.end(), want) != c.primary.end()) hit = &c;
      uint32_t lt[kMaxRows];
      int32_t lp[kMaxRows];
      std::fill(local.begin(), local.end(), -1);
      chunk_arrays(*hit, tokens, parents, local, lt, lp);
      rc = tree_forward(m, lt, lp, (int)hit->nodes.size(), prefix, 0);
      if (rc == SPEC_OK) rc = finish(m);
      if (rc != SPEC_OK) return rc;
      m->tree_window = hit->nodes;
      m->tree_window_sig = tree_signature(tokens, parents, n);
      m->cache_len = prefix + (int)hit->nodes.size();
    }
    for (int i = 0; i < n_acc; ++i) slot[i] = local[accepted[i]];
  }
  // keep = [0..prefix) ++ [prefix + ti]: the prefix is the identity, so only
  // the accepted tree rows move (quantized_llama.rs:426-433).
  int nmove = 0;
  for (int i = 0; i < n_acc; ++i) {
    const int src = prefix + slot[i], dst = prefix + i;
    if (src != dst) {
      m->idx_host[nmove] = src;
      m->idx_host[kMaxRows + nmove] = dst;
      ++nmove;
    }
  }
  if (nmove > 0) {
    cudaError_t e = cudaMemcpyAsync(m->idx_dev, m->idx_host, 2 * kMaxRows * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess)
      e = launch_kv_gather(m->kcache, m->vcache, m->cfg.n_layers, m->cfg.n_kv, m->t_max, m->cfg.head_dim, m->idx_dev,
                           m->idx_dev + kMaxRows, nmove, m->kv_tmp, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "kv reorder"));
  }
  m->cache_len = prefix + n_acc;
  for (int i = 1; i < n_acc; ++i) m->history.push_back(tokens[accepted[i]]);
  return SPEC_OK;
}

int spec_last_hidden_state(spec_model* m, float* out) {
  if (!m || !out) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "last_hidden_state with empty history");
  const uint32_t last = m->history.back();
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  const int saved = m->cache_len;
  fill_step_causal(m, &last, 1, target);
  int rc = run_forward(m, 1, F_HIDDEN);
  if (rc == SPEC_OK)
    cudaMemcpyAsync(m->hidden_host, m->hidden_out, (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost, m->stream);
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    return rc;
  }
  m->cache_len = target + 1;
  memcpy(out, m->hidden_host, (size_t)m->cfg.hidden * 4);
  return SPEC_OK;
}

int spec_observe_returning_last_hidden(spec_model* m, const uint32_t* ids, int n, float* hidden_out) {
  if (!m || !ids || !hidden_out) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (n <= 0) return m->fail(SPEC_ERR_INVALID, "observe_returning_last_hidden with empty ids");
  for (int i = 0; i < n; ++i)
    if (ids[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  // A pending last token (lazy observe) goes first.
  std::vector<uint32_t> all;
  if (!m->history.empty() && m->cache_len == (int)m->history.size() - 1) all.push_back(m->history.back());
  all.insert(all.end(), ids, ids + n);
  const int n_new = n;
  n = (int)all.size();
  ids = all.data();
  const int start = m->cache_len;
  if (start + n > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  int done = 0;
  while (done < n) {
    const int M = std::min(kMaxRows, n - done);
    fill_step_causal(m, ids + done, M, start + done);
    const bool last = done + M == n;
    int rc = run_forward(m, M, last ? F_HIDDEN : 0);
    if (rc == SPEC_OK && last)
      cudaMemcpyAsync(m->hidden_host, m->hidden_out + (size_t)(M - 1) * m->cfg.hidden, (size_t)m->cfg.hidden * 4,
                      cudaMemcpyDeviceToHost, m->stream);
    if (rc == SPEC_OK) rc = finish(m);
    if (rc != SPEC_OK) {
      m->cache_len = start;
      return rc;
    }
    done += M;
  }
  m->cache_len = start + n;
  m->history.insert(m->history.end(), ids + (n - n_new), ids + n);
  // The forward ran without the LM head, so no next-token logits are cached.
  m->last_valid = false;
  memcpy(hidden_out, m->hidden_host, (size_t)m->cfg.hidden * 4);
  return SPEC_OK;
}

int spec_apply_lm_head(spec_model* m, const float* hidden, int rows, float* out) {
  if (!m || !hidden || !out || rows < 0) return SPEC_ERR_INVALID;
  if (m->tp_size > 1) return m->fail(SPEC_ERR_UNSUPPORTED, "apply_lm_head on a tensor-parallel handle (vocabulary-parallel head)");
  DeviceGuard dg_(m->device);
  const int H = m->cfg.hidden, V = m->cfg.vocab;
  for (int r0 = 0; r0 < rows; r0 += kMaxRows) {
    const int M = std::min(kMaxRows, rows - r0);
    const int nt = nt_for_rows(M);
    cudaError_t e = cudaMemcpyAsync(m->op_in, hidden + (size_t)r0 * H, (size_t)M * H * 4, cudaMemcpyHostToDevice,
                                    m->stream);
    if (e == cudaSuccess)
      e = launch_make_operand(m->op_in, M, H, nt, m->xa, m->xa16, m->xa32, m->cfg.bf16 ? 1 : 0, m->stream);
    QmvParams p = base_params(m, m->lm, M);
    p.xfrag = m->xa;
    p.xsum16 = m->xa16;
    p.xsum32 = m->xa32;
    p.epi = EPI_STORE;
    p.out = m->logits;
    p.ld_out = V;
    if (e == cudaSuccess) e = enqueue_single(m, p, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out + (size_t)r0 * V, m->logits, (size_t)M * V * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "apply_lm_head"));
  }
  return SPEC_OK;
}

int spec_apply_lm_head_topk(spec_model* m, const float* hidden, int rows, int k, int32_t* ids_out, float* vals_out) {
  if (!m || !hidden || !ids_out || rows < 0) return SPEC_ERR_INVALID;
  if (m->tp_size > 1)
    return m->fail(SPEC_ERR_UNSUPPORTED, "apply_lm_head_topk on a tensor-parallel handle (vocabulary-parallel head)");
  if (k < 1 || k > kMaxTopK || k > m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "top-k size out of range");
  DeviceGuard dg_(m->device);
  const int H = m->cfg.hidden, V = m->cfg.vocab;
  cudaError_t e = cudaSuccess;
  if (!m->topk_part) {
    e = m->dalloc(&m->topk_part, (size_t)kMaxRows * kTopKMaxChunks * kMaxTopK * 8);
    if (e == cudaSuccess) e = m->dalloc(&m->topk_ids, (size_t)kMaxRows * kMaxTopK * 4);
    if (e == cudaSuccess) e = m->dalloc(&m->topk_vals, (size_t)kMaxRows * kMaxTopK * 4);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "top-k scratch"));
  }
  for (int r0 = 0; r0 < rows; r0 += kMaxRows) {
    const int M = std::min(kMaxRows, rows - r0);
    const int nt = nt_for_rows(M);
    e = cudaMemcpyAsync(m->op_in, hidden + (size_t)r0 * H, (size_t)M * H * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess)
      e = launch_make_operand(m->op_in, M, H, nt, m->xa, m->xa16, m->xa32, m->cfg.bf16 ? 1 : 0, m->stream);
    QmvParams p = base_params(m, m->lm, M);
    p.xfrag = m->xa;
    p.xsum16 = m->xa16;
    p.xsum32 = m->xa32;
    p.epi = EPI_STORE;
    p.out = m->logits;
    p.ld_out = V;
    if (e == cudaSuccess) e = enqueue_single(m, p, m->stream);
    if (e == cudaSuccess) e = launch_row_topk(m->logits, M, V, k, m->topk_part, m->topk_ids, m->topk_vals, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(ids_out + (size_t)r0 * k, m->topk_ids, (size_t)M * k * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess && vals_out)
      e = cudaMemcpyAsync(vals_out + (size_t)r0 * k, m->topk_vals, (size_t)M * k * 4, cudaMemcpyDeviceToHost,
                          m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "apply_lm_head_topk"));
  }
  return SPEC_OK;
}

// ---------------------------------------------------------------------------
// EAGLE draft block on the device (methods/eagle.rs:100-427, 494-575)
// ---------------------------------------------------------------------------
constexpr int kEagleMaxSteps = 64;  // draft depth (KV rows of one round)

struct EagleHead {
  Mat fc, qkv, o, gu, down;  // BF16, the checkpoint's dtype
  float* post_norm = nullptr;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  void* kcache = nullptr;    // [n_kv][kEagleMaxSteps][hd] bf16
  void* vcache = nullptr;
  float *x2 = nullptr, *h = nullptr, *t = nullptr, *h2 = nullptr, *xn = nullptr, *t2 = nullptr, *out = nullptr,
        *hin = nullptr, *logits = nullptr;
  uint32_t *xa2 = nullptr, *xa = nullptr, *xl = nullptr, *xb = nullptr, *xc = nullptr;
  float *xa2_16 = nullptr, *xa2_32 = nullptr, *xa16 = nullptr, *xa32 = nullptr, *xl16 = nullptr, *xl32 = nullptr,
        *xb16 = nullptr, *xb32 = nullptr, *xc16 = nullptr, *xc32 = nullptr;
  void* qbuf = nullptr;
  float *part_o = nullptr, *part_ml = nullptr;
  float* gpart = nullptr;
  int* gcounters = nullptr;
  FwdOp* ops = nullptr;  // fc, qkv, o, gu, down, lm
  int* done = nullptr;
  int* tok0 = nullptr;
  int* step_dev = nullptr;   // {position, slot, keys before, keys after}
  int* step_host = nullptr;  // pinned [kEagleMaxSteps][4]
  unsigned long long* anc = nullptr;
  int* ids = nullptr;
  float* vals = nullptr;
  float* lse = nullptr;
  int* ids_host = nullptr;
  float* vals_host = nullptr;
  float* lse_host = nullptr;
  int set_bf = 0;
};

namespace {

enum : int { EOP_FC = 0, EOP_QKV, EOP_O, EOP_GU, EOP_DOWN, EOP_LM, EOP_N };

// RoPE tables of the draft: eagle.rs:134-147 computes inv_freq in f32, then
// positions and inv_freq in the checkpoint dtype (BF16), their product in
// BF16, and cos/sin of that in BF16; the same roundings here.
static int eagle_rope(spec_model* m, EagleHead& e, float theta) {
  const ModelCfg& c = m->cfg;
  const int half = c.head_dim / 2, T = m->t_max + kEagleMaxSteps;
  std::vector<float> cs((size_t)T * half), sn((size_t)T * half);
  for (int i = 0; i < half; ++i) {
    const float inv = bf_round(1.f / powf(theta, (float)(2 * i) / (float)c.head_dim));
    for (int p = 0; p < T; ++p) {
      const float a = bf_round(bf_round((float)p) * inv);
      cs[(size_t)p * half + i] = bf_round(cosf(a));
      sn[(size_t)p * half + i] = bf_round(sinf(a));
    }
  }
  cudaError_t er = m->dalloc(&e.rope_cos, cs.size() * 4);
  if (er == cudaSuccess) er = m->dalloc(&e.rope_sin, sn.size() * 4);
  if (er == cudaSuccess) er = m->upload(e.rope_cos, cs.data(), cs.size() * 4);
  if (er == cudaSuccess) er = m->upload(e.rope_sin, sn.data(), sn.size() * 4);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "eagle rope tables"));
  return SPEC_OK;
}

// Buffers and the six single-op descriptors, once the matrices exist.
static int eagle_finish(spec_model* m, EagleHead& e) {
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, F = c.ffn, hd = c.head_dim, V = c.vocab, G = c.n_heads / c.n_kv;
  const int Kq = c.n_heads * hd;
  cudaError_t er = cudaSuccess;
#define EALLOC(ptr, bytes)                                                     \
  do {                                                                         \
    if (er == cudaSuccess) er = m->dalloc(&(ptr), (bytes));                    \
  } while (0)
  const size_t kv = (size_t)c.n_kv * kEagleMaxSteps * hd * 2;
  EALLOC(e.kcache, kv);
  EALLOC(e.vcache, kv);
  EALLOC(e.x2, (size_t)2 * H * 4);
  EALLOC(e.h, (size_t)H * 4);
  EALLOC(e.t, (size_t)H * 4);
  EALLOC(e.h2, (size_t)H * 4);
  EALLOC(e.xn, (size_t)H * 4);
  EALLOC(e.t2, (size_t)H * 4);
  EALLOC(e.out, (size_t)H * 4);
  EALLOC(e.hin, (size_t)H * 4);
  EALLOC(e.logits, (size_t)V * 4);
  // operands of one row: K/16 k-steps x 256 bytes (NT = 1), column sums
  auto frag = [&](uint32_t*& f, float*& s16, float*& s32, int K) {
    EALLOC(f, (size_t)K * 16);
    EALLOC(s16, (size_t)(K / 16) * 8 * 4);
    EALLOC(s32, (size_t)(K / 32) * 8 * 4);
  };
  frag(e.xa2, e.xa2_16, e.xa2_32, 2 * H);
  frag(e.xa, e.xa16, e.xa32, H);
  frag(e.xl, e.xl16, e.xl32, H);
  frag(e.xb, e.xb16, e.xb32, Kq);
  frag(e.xc, e.xc16, e.xc32, F);
  EALLOC(e.qbuf, (size_t)c.n_heads * hd * 2);
  EALLOC(e.part_o, (size_t)c.n_kv * G * hd * 4);
  EALLOC(e.part_ml, (size_t)c.n_kv * G * 2 * 4);
  size_t part = 0;
  int groups = 0;
  for (const Mat* mt : {&e.fc, &e.qkv, &e.o, &e.gu, &e.down, &m->lm}) {
    part = std::max(part, (size_t)partial_slots(*mt) * kGroupRows * 8);
    groups = std::max(groups, mt->seg[0].groups + mt->seg[1].groups);
  }
  EALLOC(e.gpart, part * 4);
  EALLOC(e.gcounters, (size_t)groups * 4);
  EALLOC(e.ops, sizeof(FwdOp) * EOP_N);
  EALLOC(e.done, sizeof(int) * EOP_N);
  EALLOC(e.tok0, 16);
  EALLOC(e.step_dev, 16);
  EALLOC(e.anc, 8);
  EALLOC(e.ids, (size_t)kEagleMaxSteps * kMaxTopK * 4);
  EALLOC(e.vals, (size_t)kEagleMaxSteps * kMaxTopK * 4);
  EALLOC(e.lse, (size_t)kEagleMaxSteps * 4);
  if (!m->topk_part) EALLOC(m->topk_part, (size_t)kMaxRows * kTopKMaxChunks * kMaxTopK * 8);
#undef EALLOC
  if (er == cudaSuccess) er = m->halloc(&e.step_host, (size_t)kEagleMaxSteps * 16);
  if (er == cudaSuccess) er = m->halloc(&e.ids_host, (size_t)kEagleMaxSteps * kMaxTopK * 4);
  if (er == cudaSuccess) er = m->halloc(&e.vals_host, (size_t)kEagleMaxSteps * kMaxTopK * 4);
  if (er == cudaSuccess) er = m->halloc(&e.lse_host, (size_t)kEagleMaxSteps * 4);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(er, "eagle buffers"));
  const unsigned long long one = 1ull;
  er = m->upload(e.anc, &one, 8);

  auto base = [&](const Mat& mt) {
    QmvParams p = base_params(m, mt, 1);
    p.part = e.gpart;
    p.counters = e.gcounters;
    p.act_bf16 = 1;
    return p;
  };
  FwdOp ops[EOP_N];
  {  // fc: concat(hidden, embedding) -> h
    QmvParams& p = ops[EOP_FC].q;
    p = base(e.fc);
    p.xfrag = e.xa2;
    p.xsum16 = e.xa2_16;
    p.xsum32 = e.xa2_32;
    p.epi = EPI_STORE;
    p.out = e.h;
    p.ld_out = H;
  }
  {  // q, k, v with RoPE; K/V rows into the draft's cache (no input norm)
    QmvParams& p = ops[EOP_QKV].q;
    p = base(e.qkv);
    p.xfrag = e.xa;
    p.xsum16 = e.xa16;
    p.xsum32 = e.xa32;
    p.epi = EPI_QKV;
    p.n_q_heads = c.n_heads;
    p.n_kv_heads = c.n_kv;
    p.head_dim = hd;
    p.rope_interleaved = 0;  // candle_nn::rotary_emb::rope (rotate-half)
    p.rope_cos = e.rope_cos;
    p.rope_sin = e.rope_sin;
    p.positions = e.step_dev;
    p.kv_slots = e.step_dev + 1;
    p.qbuf = e.qbuf;
    p.kcache = e.kcache;
    p.vcache = e.vcache;
    p.t_max = kEagleMaxSteps;
  }
  {  // o_proj -> t
    QmvParams& p = ops[EOP_O].q;
    p = base(e.o);
    p.xfrag = e.xb;
    p.xsum16 = e.xb16;
    p.xsum32 = e.xb32;
    p.epi = EPI_STORE;
    p.out = e.t;
    p.ld_out = H;
  }
  {  // gate/up -> silu(g) * u as the down operand
    QmvParams& p = ops[EOP_GU].q;
    p = base(e.gu);
    p.xfrag = e.xa;
    p.xsum16 = e.xa16;
    p.xsum32 = e.xa32;
    p.epi = EPI_SILU;
    p.next_frag = e.xc;
    p.next_xsum16 = e.xc16;
    p.next_xsum32 = e.xc32;
  }
  {  // down -> t2
    QmvParams& p = ops[EOP_DOWN].q;
    p = base(e.down);
    p.xfrag = e.xc;
    p.xsum16 = e.xc16;
    p.xsum32 = e.xc32;
    p.epi = EPI_STORE;
    p.out = e.t2;
    p.ld_out = H;
  }
  {  // the target's LM head -> logits row
    QmvParams& p = ops[EOP_LM].q;
    p = base(m->lm);
    p.act_bf16 = c.bf16 ? 1 : 0;
    p.xfrag = e.xl;
    p.xsum16 = e.xl16;
    p.xsum32 = e.xl32;
    p.epi = EPI_STORE;
    p.out = e.logits;
    p.ld_out = V;
  }
  for (auto& op : ops) op.dep = -1;
  if (er == cudaSuccess) er = m->upload(e.ops, ops, sizeof(ops));
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "eagle descriptors"));
  e.set_bf = fwd_fmt_set_for(fmt_bit(WF_BF16));
  return SPEC_OK;
}

static int eagle_build(spec_model* m, const Part& fc, const Part& q, const Part& k, const Part& v, const Part& o,
                const Part& g, const Part& u, const Part& d, float theta, std::shared_ptr<EagleHead>& out) {
  const ModelCfg& c = m->cfg;
  auto e = std::make_shared<EagleHead>();
  const int saved_bits = m->fmt_bits;  // the draft's BF16 does not join the target's format set
  int rc = build_mat(m, {fc}, 2 * c.hidden, false, e->fc);
  if (rc == SPEC_OK) rc = build_mat(m, {q, k, v}, c.hidden, false, e->qkv);
  if (rc == SPEC_OK) rc = build_mat(m, {o}, c.n_heads * c.head_dim, false, e->o);
  if (rc == SPEC_OK) rc = build_mat(m, {g, u}, c.hidden, true, e->gu);
  if (rc == SPEC_OK) rc = build_mat(m, {d}, c.ffn, false, e->down);
  m->fmt_bits = saved_bits;
  if (rc == SPEC_OK) rc = eagle_rope(m, *e, theta);
  if (rc == SPEC_OK) rc = eagle_finish(m, *e);
  if (rc == SPEC_OK) out = e;
  return rc;
}

static int eagle_check_target(spec_model* m) {
  const ModelCfg& c = m->cfg;
  if (m->tp_size > 1) return m->fail(SPEC_ERR_UNSUPPORTED, "EAGLE draft on a tensor-parallel handle");
  if ((2 * c.hidden) % 128 || c.hidden % 128 || c.ffn % 128 || (c.n_heads * c.head_dim) % 128)
    return m->fail(SPEC_ERR_UNSUPPORTED, "EAGLE draft shapes are not multiples of 128");
  return SPEC_OK;
}

}  // namespace

int spec_eagle_attach(spec_model* m, const spec_eagle_weights* w) {
  if (!m || !w || !w->fc || !w->q || !w->k || !w->v || !w->o || !w->gate || !w->up || !w->down || !w->post_norm)
    return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (int rc = eagle_check_target(m)) return rc;
  const ModelCfg& c = m->cfg;
  const int hd = c.head_dim;
  auto host = [](const void* src, int rows) {
    Part p;
    p.src = static_cast<const uint8_t*>(src);
    p.on_device = false;
    p.fmt = WF_BF16;
    p.rows = rows;
    return p;
  };
  std::shared_ptr<EagleHead> e;
  int rc = eagle_build(m, host(w->fc, c.hidden), host(w->q, c.n_heads * hd), host(w->k, c.n_kv * hd),
                       host(w->v, c.n_kv * hd), host(w->o, c.hidden), host(w->gate, c.ffn), host(w->up, c.ffn),
                       host(w->down, c.hidden), w->rope_theta > 0.f ? w->rope_theta : c.rope_theta, e);
  if (rc != SPEC_OK) return rc;
  cudaError_t er = m->dalloc(&e->post_norm, (size_t)c.hidden * 4);
  if (er == cudaSuccess) er = m->upload(e->post_norm, w->post_norm, (size_t)c.hidden * 4);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "eagle norm"));
  m->eagle = e;
  return SPEC_OK;
}

int spec_eagle_attach_synthetic(spec_model* m, uint64_t seed) {
  if (!m) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (int rc = eagle_check_target(m)) return rc;
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, hd = c.head_dim, F = c.ffn;
  std::vector<void*> temps;
  uint64_t st = seed * 0x9E3779B97F4A7C15ull + 0xEA61Eull;
  auto tseed = [&]() { return st += 0x632BE59BD9B4E019ull; };
  Part fc, q, k, v, o, g, u, d;
  int rc = synth_part(m, temps, WF_BF16, H, 2 * H, tseed(), fc);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, c.n_heads * hd, H, tseed(), q);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, c.n_kv * hd, H, tseed(), k);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, c.n_kv * hd, H, tseed(), v);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, H, c.n_heads * hd, tseed(), o);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, F, H, tseed(), g);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, F, H, tseed(), u);
  if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, H, F, tseed(), d);
  std::shared_ptr<EagleHead> e;
  if (rc == SPEC_OK) rc = eagle_build(m, fc, q, k, v, o, g, u, d, c.rope_theta, e);
  if (rc == SPEC_OK) rc = synth_vec(m, &e->post_norm, H, tseed(), 1.f);
  cudaStreamSynchronize(m->stream);
  for (void* t : temps) cudaFree(t);
  if (rc != SPEC_OK) return rc;
  m->eagle = e;
  return SPEC_OK;
}

int spec_eagle_draft(spec_model* m, const float* hidden, uint32_t root, int position, int depth, int k,
                     int32_t* ids_out, float* logprobs_out) {
  if (!m || !hidden || !ids_out || depth < 1) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  EagleHead* e = m->eagle.get();
  if (!e) return m->fail(SPEC_ERR_INVALID, "no EAGLE draft attached (spec_eagle_attach)");
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, V = c.vocab, G = c.n_heads / c.n_kv;
  if (depth > kEagleMaxSteps) return m->fail(SPEC_ERR_UNSUPPORTED, "EAGLE draft depth above 64");
  if (k < 1 || k > kMaxTopK || k > V) return m->fail(SPEC_ERR_INVALID, "top-k size out of range");
  if (root >= (uint32_t)V) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  if (position < 0 || position + depth > m->t_max + kEagleMaxSteps)
    return m->fail(SPEC_ERR_INVALID, "EAGLE draft position outside the RoPE table");
  cudaStream_t s = m->stream;
  for (int i = 0; i < depth; ++i) {
    e->step_host[4 * i + 0] = position + i;  // RoPE position (eagle.rs:544: history_len + step)
    e->step_host[4 * i + 1] = i;             // KV row: the cache holds this round only (draft.reset())
    e->step_host[4 * i + 2] = i;             // keys before this row
    e->step_host[4 * i + 3] = i + 1;
  }
  const int root_i = (int)root;
  cudaError_t er = cudaMemcpyAsync(e->hin, hidden, (size_t)H * 4, cudaMemcpyHostToDevice, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(e->tok0, &root_i, 4, cudaMemcpyHostToDevice, s);
  if (er == cudaSuccess) er = cudaMemsetAsync(m->err_dev, 0, 16, s);
  auto gemv = [&](int op, int set) {
    FwdParams fp;
    fp.ops = e->ops + op;
    fp.n_ops = 1;
    fp.done = e->done + op;
    fp.err = m->err_dev;
    return launch_fwd(fp, set, 1, s, false);
  };
  AttnParams a;
  a.q = e->qbuf;
  a.kcache = e->kcache;
  a.vcache = e->vcache;
  a.n_kv = c.n_kv;
  a.G = G;
  a.hd = c.head_dim;
  a.M = 1;
  a.t_max = kEagleMaxSteps;
  a.step = e->step_dev + 2;
  a.anc = e->anc;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)c.head_dim);
  a.chunk = kEagleMaxSteps;
  a.max_splits = 1;
  a.part_o = e->part_o;
  a.part_ml = e->part_ml;
  a.frag = e->xb;
  a.xsum16 = e->xb16;
  a.xsum32 = e->xb32;
  a.act_bf16 = 1;
  a.err = m->err_dev;
  for (int i = 0; i < depth && er == cudaSuccess; ++i) {
    const float* hid = i == 0 ? e->hin : e->out;
    const int* tok = i == 0 ? e->tok0 : e->ids + (size_t)(i - 1) * k;  // previous step's top-1
    er = cudaMemcpyAsync(e->step_dev, e->step_host + 4 * i, 16, cudaMemcpyHostToDevice, s);
    if (er == cudaSuccess) er = launch_eagle_concat(m->embed_raw, m->embed_fmt, H, V, tok, hid, e->x2, m->err_dev, s);
    if (er == cudaSuccess) er = launch_make_operand(e->x2, 1, 2 * H, 1, e->xa2, e->xa2_16, e->xa2_32, 1, s);
    if (er == cudaSuccess) er = gemv(EOP_FC, e->set_bf);
    if (er == cudaSuccess) er = launch_make_operand(e->h, 1, H, 1, e->xa, e->xa16, e->xa32, 1, s);
    if (er == cudaSuccess) er = gemv(EOP_QKV, e->set_bf);
    if (er == cudaSuccess) er = launch_attention(a, 1, s, false);
    if (er == cudaSuccess) er = gemv(EOP_O, e->set_bf);
    if (er == cudaSuccess) er = launch_eagle_resid_norm(e->t, e->h, e->post_norm, H, c.eps, e->h2, e->xn, s);
    if (er == cudaSuccess) er = launch_make_operand(e->xn, 1, H, 1, e->xa, e->xa16, e->xa32, 1, s);
    if (er == cudaSuccess) er = gemv(EOP_GU, e->set_bf);
    if (er == cudaSuccess) er = gemv(EOP_DOWN, e->set_bf);
    if (er == cudaSuccess) er = launch_eagle_add(e->t2, e->h2, e->out, H, s);
    if (er == cudaSuccess) er = launch_make_operand(e->out, 1, H, 1, e->xl, e->xl16, e->xl32, c.bf16 ? 1 : 0, s);
    if (er == cudaSuccess) er = gemv(EOP_LM, m->fmt_set);
    if (er == cudaSuccess)
      er = launch_row_topk(e->logits, 1, V, k, m->topk_part, e->ids + (size_t)i * k, e->vals + (size_t)i * k, s);
    if (er == cudaSuccess) er = launch_row_lse(e->logits, V, e->lse + i, s);
  }
  if (er == cudaSuccess)
    er = cudaMemcpyAsync(e->ids_host, e->ids, (size_t)depth * k * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess)
    er = cudaMemcpyAsync(e->vals_host, e->vals, (size_t)depth * k * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(e->lse_host, e->lse, (size_t)depth * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(m->err_host, m->err_dev, 16, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaStreamSynchronize(s);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "eagle draft"));
  if (m->err_host[0]) return m->fail(SPEC_ERR_TIMEOUT, "device error during the EAGLE draft");
  memcpy(ids_out, e->ids_host, (size_t)depth * k * 4);
  if (logprobs_out)  // eagle.rs:557-559: logits[i] - lse
    for (int i = 0; i < depth * k; ++i) logprobs_out[i] = e->vals_host[i] - e->lse_host[i / k];
  return SPEC_OK;
}

// ---------------------------------------------------------------------------
// Medusa draft heads on the device (methods/medusa.rs:509-584, 706-734)
// ---------------------------------------------------------------------------
struct MedusaHeads {
  int n_heads = 0, layers = 0;
  std::vector<Mat> res;        // [head][layer] BF16 [H][H]
  std::vector<float*> res_b;   // [head][layer] f32 [H]
  std::vector<Mat> out;        // [head] BF16 [V][H]
  float *hin = nullptr, *x = nullptr, *y = nullptr, *logits = nullptr;
  uint32_t* xa = nullptr;
  float *xa16 = nullptr, *xa32 = nullptr;
  float* gpart = nullptr;
  int* gcounters = nullptr;
  FwdOp* ops = nullptr;        // [head][layer] residual linears, then [head] output projections
  int* done = nullptr;
  int* ids = nullptr;
  float* vals = nullptr;
  float* lse = nullptr;
  int* ids_host = nullptr;
  float* vals_host = nullptr;
  float* lse_host = nullptr;
  int set_bf = 0;
};

namespace {

constexpr int kMedusaMaxHeads = 8;
constexpr int kMedusaMaxLayers = 4;

static int medusa_check(spec_model* m, int n_heads, int layers) {
  const ModelCfg& c = m->cfg;
  if (n_heads < 1 || n_heads > kMedusaMaxHeads || layers < 0 || layers > kMedusaMaxLayers)
    return m->fail(SPEC_ERR_INVALID, "Medusa heads: 1..8 heads of 0..4 residual layers");
  if (m->tp_size > 1) return m->fail(SPEC_ERR_UNSUPPORTED, "Medusa heads on a tensor-parallel handle");
  if (c.hidden % 128 || c.vocab % 128) return m->fail(SPEC_ERR_UNSUPPORTED, "Medusa head shapes are not multiples of 128");
  return SPEC_OK;
}

// Builds the heads' matrices from parts ([head][layer] residual weights, then
// [head] output projections) and their buffers and op descriptors.
static int medusa_build(spec_model* m, int n_heads, int layers, const std::vector<Part>& res, const std::vector<Part>& outp,
                 std::shared_ptr<MedusaHeads>& out) {
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, V = c.vocab;
  auto h = std::make_shared<MedusaHeads>();
  h->n_heads = n_heads;
  h->layers = layers;
  h->res.resize((size_t)n_heads * layers);
  h->res_b.assign((size_t)n_heads * layers, nullptr);
  h->out.resize(n_heads);
  const int saved_bits = m->fmt_bits;  // the heads' BF16 does not join the target's format set
  int rc = SPEC_OK;
  for (size_t i = 0; i < h->res.size() && rc == SPEC_OK; ++i) rc = build_mat(m, {res[i]}, H, false, h->res[i]);
  for (int i = 0; i < n_heads && rc == SPEC_OK; ++i) rc = build_mat(m, {outp[i]}, H, false, h->out[i]);
  m->fmt_bits = saved_bits;
  if (rc != SPEC_OK) return rc;
  cudaError_t er = cudaSuccess;
#define MALLOC(ptr, bytes)                                                     \
  do {                                                                         \
    if (er == cudaSuccess) er = m->dalloc(&(ptr), (bytes));                    \
  } while (0)
  MALLOC(h->hin, (size_t)H * 4);
  MALLOC(h->x, (size_t)H * 4);
  MALLOC(h->y, (size_t)H * 4);
  MALLOC(h->logits, (size_t)V * 4);
  MALLOC(h->xa, (size_t)H * 16);  // one row's operand: H/16 k-steps x 256 bytes (NT = 1)
  MALLOC(h->xa16, (size_t)(H / 16) * 8 * 4);
  MALLOC(h->xa32, (size_t)(H / 32) * 8 * 4);
  size_t part = 0;
  int groups = 0;
  for (const auto* v : {&h->res, &h->out})
    for (const Mat& mt : *v) {
      part = std::max(part, (size_t)partial_slots(mt) * kGroupRows * 8);
      groups = std::max(groups, mt.seg[0].groups + mt.seg[1].groups);
    }
  MALLOC(h->gpart, part * 4);
  MALLOC(h->gcounters, (size_t)groups * 4);
  const int n_ops = n_heads * (layers + 1);
  MALLOC(h->ops, sizeof(FwdOp) * n_ops);
  MALLOC(h->done, sizeof(int) * n_ops);
  MALLOC(h->ids, (size_t)n_heads * kMaxTopK * 4);
  MALLOC(h->vals, (size_t)n_heads * kMaxTopK * 4);
  MALLOC(h->lse, (size_t)n_heads * 4);
  if (!m->topk_part) MALLOC(m->topk_part, (size_t)kMaxRows * kTopKMaxChunks * kMaxTopK * 8);
#undef MALLOC
  if (er == cudaSuccess) er = m->halloc(&h->ids_host, (size_t)n_heads * kMaxTopK * 4);
  if (er == cudaSuccess) er = m->halloc(&h->vals_host, (size_t)n_heads * kMaxTopK * 4);
  if (er == cudaSuccess) er = m->halloc(&h->lse_host, (size_t)n_heads * 4);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(er, "Medusa buffers"));
  h->set_bf = fwd_fmt_set_for(fmt_bit(WF_BF16));
  out = h;
  // The caller fills the residual biases (res_b), then uploads the op
  // descriptors (medusa_upload_ops).
  return SPEC_OK;
}

static int medusa_upload_ops(spec_model* m, MedusaHeads& h) {
  const int n_ops = h.n_heads * (h.layers + 1);
  std::vector<FwdOp> ops(n_ops);
  const ModelCfg& c = m->cfg;
  for (int i = 0; i < n_ops; ++i) {
    const bool res = i < h.n_heads * h.layers;
    const Mat& mt = res ? h.res[i] : h.out[i - h.n_heads * h.layers];
    QmvParams p = base_params(m, mt, 1);
    p.part = h.gpart;
    p.counters = h.gcounters;
    p.act_bf16 = 1;
    p.xfrag = h.xa;
    p.xsum16 = h.xa16;
    p.xsum32 = h.xa32;
    p.epi = EPI_STORE;
    p.out = res ? h.y : h.logits;
    p.ld_out = res ? c.hidden : c.vocab;
    p.bias = res ? h.res_b[i] : nullptr;
    ops[i].q = p;
    ops[i].dep = -1;
  }
  cudaError_t er = m->upload(h.ops, ops.data(), sizeof(FwdOp) * n_ops);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "Medusa descriptors"));
  return SPEC_OK;
}

}  // namespace

int spec_medusa_attach(spec_model* m, const spec_medusa_weights* w) {
  if (!m || !w || (w->residual_layers > 0 && (!w->res_w || !w->res_b)) || !w->out_w) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (int rc = medusa_check(m, w->n_heads, w->residual_layers)) return rc;
  const ModelCfg& c = m->cfg;
  const int n_res = w->n_heads * w->residual_layers;
  for (int i = 0; i < n_res; ++i)
    if (!w->res_w[i] || !w->res_b[i]) return SPEC_ERR_INVALID;
  for (int i = 0; i < w->n_heads; ++i)
    if (!w->out_w[i]) return SPEC_ERR_INVALID;
  auto host = [](const void* src, int rows) {
    Part p;
    p.src = static_cast<const uint8_t*>(src);
    p.on_device = false;
    p.fmt = WF_BF16;
    p.rows = rows;
    return p;
  };
  std::vector<Part> res, outp;
  for (int i = 0; i < n_res; ++i) res.push_back(host(w->res_w[i], c.hidden));
  for (int i = 0; i < w->n_heads; ++i) outp.push_back(host(w->out_w[i], c.vocab));
  std::shared_ptr<MedusaHeads> h;
  int rc = medusa_build(m, w->n_heads, w->residual_layers, res, outp, h);
  if (rc != SPEC_OK) return rc;
  for (int i = 0; i < n_res; ++i) {
    cudaError_t er = m->dalloc(&h->res_b[i], (size_t)c.hidden * 4);
    if (er == cudaSuccess) er = m->upload(h->res_b[i], w->res_b[i], (size_t)c.hidden * 4);
    if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "Medusa biases"));
  }
  if ((rc = medusa_upload_ops(m, *h)) != SPEC_OK) return rc;
  m->medusa = h;
  return SPEC_OK;
}

int spec_medusa_attach_synthetic(spec_model* m, int n_heads, int residual_layers, uint64_t seed) {
  if (!m) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (int rc = medusa_check(m, n_heads, residual_layers)) return rc;
  const ModelCfg& c = m->cfg;
  std::vector<void*> temps;
  uint64_t st = seed * 0x9E3779B97F4A7C15ull + 0x3ED05Aull;
  auto tseed = [&]() { return st += 0x632BE59BD9B4E019ull; };
  std::vector<Part> res(n_heads * residual_layers), outp(n_heads);
  int rc = SPEC_OK;
  for (auto& p : res)
    if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, c.hidden, c.hidden, tseed(), p);
  for (auto& p : outp)
    if (rc == SPEC_OK) rc = synth_part(m, temps, WF_BF16, c.vocab, c.hidden, tseed(), p);
  std::shared_ptr<MedusaHeads> h;
  if (rc == SPEC_OK) rc = medusa_build(m, n_heads, residual_layers, res, outp, h);
  for (int i = 0; rc == SPEC_OK && i < n_heads * residual_layers; ++i)
    rc = synth_vec(m, &h->res_b[i], c.hidden, tseed(), 0.f);
  cudaStreamSynchronize(m->stream);
  for (void* t : temps) cudaFree(t);
  if (rc == SPEC_OK) rc = medusa_upload_ops(m, *h);
  if (rc != SPEC_OK) return rc;
  m->medusa = h;
  return SPEC_OK;
}

int spec_medusa_topk(spec_model* m, const float* hidden, int k, int32_t* ids_out, float* logprobs_out) {
  if (!m || !hidden || !ids_out) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  MedusaHeads* h = m->medusa.get();
  if (!h) return m->fail(SPEC_ERR_INVALID, "no Medusa heads attached (spec_medusa_attach)");
  const ModelCfg& c = m->cfg;
  const int H = c.hidden, V = c.vocab;
  if (k < 1 || k > kMaxTopK || k > V) return m->fail(SPEC_ERR_INVALID, "top-k size out of range");
  cudaStream_t s = m->stream;
  cudaError_t er = cudaMemcpyAsync(h->hin, hidden, (size_t)H * 4, cudaMemcpyHostToDevice, s);
  if (er == cudaSuccess) er = cudaMemsetAsync(m->err_dev, 0, 16, s);
  auto gemv = [&](int op) {
    FwdParams fp;
    fp.ops = h->ops + op;
    fp.n_ops = 1;
    fp.done = h->done + op;
    fp.err = m->err_dev;
    return launch_fwd(fp, h->set_bf, 1, s, false);
  };
  // Every head reads the same hidden row (medusa.rs:706-708).
  for (int hd = 0; hd < h->n_heads && er == cudaSuccess; ++hd) {
    const float* x = h->hin;
    for (int l = 0; l < h->layers && er == cudaSuccess; ++l) {
      // x' = x + SiLU(W x + b) (medusa.rs:571-575)
      er = launch_make_operand(x, 1, H, 1, h->xa, h->xa16, h->xa32, 1, s);
      if (er == cudaSuccess) er = gemv(hd * h->layers + l);
      if (er == cudaSuccess) er = launch_medusa_res(x, h->y, h->x, H, s);
      x = h->x;
    }
    if (er == cudaSuccess) er = launch_make_operand(x, 1, H, 1, h->xa, h->xa16, h->xa32, 1, s);
    if (er == cudaSuccess) er = gemv(h->n_heads * h->layers + hd);
    // top_k_indices over the head's logits (medusa.rs:713-734, 477-487)
    if (er == cudaSuccess)
      er = launch_row_topk(h->logits, 1, V, k, m->topk_part, h->ids + (size_t)hd * k, h->vals + (size_t)hd * k, s);
    if (er == cudaSuccess) er = launch_row_lse(h->logits, V, h->lse + hd, s);
  }
  const int n = h->n_heads;
  if (er == cudaSuccess) er = cudaMemcpyAsync(h->ids_host, h->ids, (size_t)n * k * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(h->vals_host, h->vals, (size_t)n * k * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(h->lse_host, h->lse, (size_t)n * 4, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaMemcpyAsync(m->err_host, m->err_dev, 16, cudaMemcpyDeviceToHost, s);
  if (er == cudaSuccess) er = cudaStreamSynchronize(s);
  if (er != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(er, "Medusa heads"));
  if (m->err_host[0]) return m->fail(SPEC_ERR_TIMEOUT, "device error during the Medusa heads");
  memcpy(ids_out, h->ids_host, (size_t)n * k * 4);
  if (logprobs_out)
    for (int i = 0; i < n * k; ++i) logprobs_out[i] = h->vals_host[i] - h->lse_host[i / k];
  return SPEC_OK;
}

int spec_medusa_num_heads(const spec_model* m) { return (m && m->medusa) ? m->medusa->n_heads : 0; }

int spec_embed_tokens(spec_model* m, const uint32_t* ids, int n, float* out) {
  if (!m || !ids || !out || n < 0) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  const int H = m->cfg.hidden;
  for (int i = 0; i < n; ++i)
    if (ids[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  for (int r0 = 0; r0 < n; r0 += kMaxRows) {
    const int M = std::min(kMaxRows, n - r0);
    for (int i = 0; i < M; ++i) m->step_host->tokens[i] = (int)ids[r0 + i];
    cudaError_t e = cudaMemcpyAsync(m->step_dev, m->step_host, sizeof(StepDev), cudaMemcpyHostToDevice, m->stream);
    EmbedParams ep;
    ep.table = m->embed_raw;
    ep.fmt = m->embed_fmt;
    ep.H = H;
    ep.V = m->cfg.vocab;
    ep.M = M;
    ep.tokens = m->step_dev->tokens;
    ep.h = m->op_in;
    ep.ss_out = m->ss;
    ep.norm = nullptr;
    // Scratch operand, not consumed: the H-wide one (the O-projection
    // operand may be narrower than H, and its zero columns must stay zero).
    ep.frag = m->xa;
    ep.xsum16 = m->xa16;
    ep.xsum32 = m->xa32;
    ep.act_bf16 = m->cfg.bf16 ? 1 : 0;
    ep.err = m->err_dev;
    if (e == cudaSuccess) e = launch_embed(ep, nt_for_rows(M), m->stream, false);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out + (size_t)r0 * H, m->op_in, (size_t)M * H * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "embed_tokens"));
  }
  return SPEC_OK;
}

int spec_last_hidden_states_multi(spec_model* m, const int32_t* layers, int n_sel, float* final_out,
                                  float* layer_outs) {
  if (!m || !final_out || n_sel < 0 || (n_sel > 0 && (!layers || !layer_outs))) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "last_hidden_states_multi with empty history");
  for (int i = 0; i < n_sel; ++i)
    if (layers[i] < 0 || layers[i] >= m->cfg.n_layers)
      return m->fail(SPEC_ERR_INVALID, "collect_layers[" + std::to_string(i) + "] = " + std::to_string(layers[i]) +
                                           " out of range (n_layers=" + std::to_string(m->cfg.n_layers) + ")");
  const int H = m->cfg.hidden;
  if (!m->collect) {
    cudaError_t e = m->dalloc(&m->collect, (size_t)m->cfg.n_layers * H * 4);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "collect buffer"));
  }
  const uint32_t last = m->history.back();
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  std::vector<int> sel(layers, layers + n_sel);
  fill_step_causal(m, &last, 1, target);
  const int saved = m->cache_len;
  int rc = run_forward(m, 1, F_HIDDEN, &sel);
  if (rc == SPEC_OK)
    cudaMemcpyAsync(m->hidden_host, m->hidden_out, (size_t)H * 4, cudaMemcpyDeviceToHost, m->stream);
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    return rc;
  }
  memcpy(final_out, m->hidden_host, (size_t)H * 4);
  if (n_sel > 0) {
    cudaError_t e = cudaMemcpy(layer_outs, m->collect, (size_t)n_sel * H * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "collect copy"));
  }
  m->cache_len = target + 1;
  return SPEC_OK;
}

int spec_verify_greedy(spec_model* m, const uint32_t* drafts, int k, int* n_accepted, uint32_t* next_token,
                       int32_t* argmax_out) {
  if (!m || !n_accepted || !next_token || k < 0 || (k > 0 && !drafts)) return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "batched_logits with empty history");
  if (k + 1 > kMaxRows) return m->fail(SPEC_ERR_UNSUPPORTED, "k+1 exceeds SPEC_MAX_ROWS");
  for (int i = 0; i < k; ++i)
    if (drafts[i] >= (uint32_t)m->cfg.vocab) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  const int saved = m->cache_len;
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  if (target + k + 1 > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  std::vector<uint32_t> combined(k + 1);
  combined[0] = m->history.back();
  if (k) memcpy(combined.data() + 1, drafts, (size_t)k * 4);
  fill_step_causal(m, combined.data(), k + 1, target);
  int rc = run_forward(m, k + 1, F_LOGITS);
  if (rc == SPEC_OK) {
    cudaError_t e = launch_row_argmax(m->logits, k + 1, m->cfg.vocab, m->argmax_dev, nullptr,
                                      m->argmax_slots, m->argmax_counters, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(m->argmax_host, m->argmax_dev, (size_t)(k + 1) * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "argmax"));
  }
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    return rc;
  }
  m->cache_len = target + k + 1;
  m->last_valid = true;
  m->history.insert(m->history.end(), drafts, drafts + k);
  int acc = 0;
  while (acc < k && (uint32_t)m->argmax_host[acc] == drafts[acc]) ++acc;
  *n_accepted = acc;
  *next_token = (uint32_t)m->argmax_host[acc];
  if (argmax_out) memcpy(argmax_out, m->argmax_host, (size_t)(k + 1) * 4);
  return SPEC_OK;
}

// One greedy vanilla SD round (methods/vanilla.rs:285-369 at temperature 0)
// over two handles, natively: k draft steps (device argmax of the draft's
// next-token row, then a lazy observe), one target verify with the device
// accept walk, then both handles roll back to the accepted prefix and
// observe the token that follows it.  Same calls, same order and same
// results as issuing them one by one through the ABI.
int spec_sd_greedy_round(spec_model* target, spec_model* draft, int k, uint32_t* commits_out, int* n_out) {
  if (!target || !draft || !commits_out || !n_out || k < 0 || k + 1 > kMaxRows) return SPEC_ERR_INVALID;
  if (target->history.size() != draft->history.size())
    return target->fail(SPEC_ERR_INVALID, "target and draft histories differ in length");
  const int pre = (int)target->history.size();
  uint32_t drafts[kMaxRows];
  for (int i = 0; i < k; ++i) {
    int acc;
    uint32_t nxt;
    int rc = spec_verify_greedy(draft, nullptr, 0, &acc, &nxt, nullptr);
    if (rc == SPEC_OK) rc = spec_observe(draft, &nxt, 1);
    if (rc != SPEC_OK) {
      if (draft != target) target->err = draft->err;
      return rc;
    }
    drafts[i] = nxt;
  }
  int n_acc = 0;
  uint32_t bonus = 0;
  int rc = spec_verify_greedy(target, drafts, k, &n_acc, &bonus, nullptr);
  if (rc == SPEC_OK) rc = spec_rollback_to(target, pre + n_acc);
  if (rc == SPEC_OK) rc = spec_observe(target, &bonus, 1);
  if (rc == SPEC_OK) rc = spec_rollback_to(draft, pre + n_acc);
  if (rc == SPEC_OK) rc = spec_observe(draft, &bonus, 1);
  if (rc != SPEC_OK) return rc;
  for (int i = 0; i < n_acc; ++i) commits_out[i] = drafts[i];
  commits_out[n_acc] = bonus;
  *n_out = n_acc + 1;
  return SPEC_OK;
}

// spec_verify_rejection with the draft rows either on the host (draft_probs)
// or already in m->rej_q (draft_probs null; the sampled round puts them
// there on the device).
int verify_rejection_core(spec_model* m, const uint32_t* drafts, int k, const float* draft_probs, float temperature,
                          const float* uniforms, int n_uniforms, int budget, uint32_t* commits, int* n_commits,
                          int* n_uniforms_used) {
  DeviceGuard dg_(m->device);
  if (!std::isfinite(temperature) || temperature < 0.f) return m->fail(SPEC_ERR_INVALID, "invalid temperature");
  if (budget < 1) return m->fail(SPEC_ERR_INVALID, "token budget must be >= 1");
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "batched_logits with empty history");
  if (k + 1 > kMaxRows) return m->fail(SPEC_ERR_UNSUPPORTED, "k+1 exceeds SPEC_MAX_ROWS");
  const int V = m->cfg.vocab;
  for (int i = 0; i < k; ++i)
    if (drafts[i] >= (uint32_t)V) return m->fail(SPEC_ERR_INVALID, "token id out of range");
  const int saved = m->cache_len;
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  if (target + k + 1 > m->t_max) return m->fail(SPEC_ERR_INVALID, "KV capacity exceeded");
  std::vector<uint32_t> combined(k + 1);
  combined[0] = m->history.back();
  if (k) memcpy(combined.data() + 1, drafts, (size_t)k * 4);
  // Stage the round's inputs before the forward (every call ends with its
  // stream drained, so the pinned slots are free) so their upload overlaps it.
  RejStep* st = m->rej_step_host;
  st->k = k;
  st->budget = budget;
  st->n_uniforms = std::min(n_uniforms, kMaxRows + 1);
  for (int i = 0; i < k; ++i) st->drafts[i] = (int)drafts[i];
  for (int i = 0; i < st->n_uniforms; ++i) st->uniforms[i] = uniforms[i];
  if (k && draft_probs) memcpy(m->rej_q_host, draft_probs, (size_t)k * V * 4);
  cudaError_t e0 = cudaSuccess;
  if (k && draft_probs)
    e0 = cudaMemcpyAsync(m->rej_q, m->rej_q_host, (size_t)k * V * 4, cudaMemcpyHostToDevice, m->stream);
  if (e0 == cudaSuccess)
    e0 = cudaMemcpyAsync(m->rej_step_dev, st, sizeof(RejStep), cudaMemcpyHostToDevice, m->stream);
  if (e0 != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e0, "rejection inputs"));
  fill_step_causal(m, combined.data(), k + 1, target);
  int rc = run_forward(m, k + 1, F_LOGITS);
  if (rc == SPEC_OK) {
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = cudaMemsetAsync(m->rej_out_dev, 0, (4 + kMaxRows) * 4, m->stream);
    if (e == cudaSuccess)
      e = launch_rejection(m->logits, m->rej_q, m->rej_r, m->rej_step_dev, k, V, temperature, m->rej_out_dev,
                           m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(m->rej_out_host, m->rej_out_dev, (4 + kMaxRows) * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "rejection sampling"));
  }
  if (rc == SPEC_OK) rc = finish(m);
  if (rc == SPEC_OK && m->rej_out_host[2] != REJ_OK) {
    static const char* msgs[] = {"", "softmax produced non-positive sum", "adjusted distribution has non-positive mass",
                                 "not enough uniforms for the round", "invalid distribution"};
    const int st = m->rej_out_host[2];
    rc = m->fail(SPEC_ERR_INVALID, st > 0 && st < 5 ? msgs[st] : "sampling error");
  }
  if (rc != SPEC_OK) {
    m->cache_len = saved;
    return rc;
  }
  m->cache_len = target + k + 1;
  m->last_valid = true;
  m->history.insert(m->history.end(), drafts, drafts + k);
  const int n = m->rej_out_host[0];
  for (int i = 0; i < n; ++i) commits[i] = (uint32_t)m->rej_out_host[4 + i];
  *n_commits = n;
  if (n_uniforms_used) *n_uniforms_used = m->rej_out_host[1];
  return SPEC_OK;
}

int spec_verify_rejection(spec_model* m, const uint32_t* drafts, int k, const float* draft_probs,
                          float temperature, const float* uniforms, int n_uniforms, int budget, uint32_t* commits,
                          int* n_commits, int* n_uniforms_used) {
  if (!m || !commits || !n_commits || k < 0 || (k > 0 && (!drafts || !draft_probs)) || n_uniforms < 0 ||
      (n_uniforms > 0 && !uniforms))
    return SPEC_ERR_INVALID;
  return verify_rejection_core(m, drafts, k, draft_probs, temperature, uniforms, n_uniforms, budget, commits,
                               n_commits, n_uniforms_used);
}

// ---------------------------------------------------------------------------
// The reference's seeded sampling stream (rand 0.8 StdRng, restated from the
// published algorithms; see include/spec_b200.h) and the sampled SD round.
// ---------------------------------------------------------------------------
struct spec_rng {
  uint32_t key[8];
  uint64_t block = 0;  // counter of the next block to generate
  uint32_t buf[64];    // four blocks, as rand_chacha buffers them (the order is the stream's)
  int pos = 64;
};

namespace {

inline uint32_t rotl32(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

// One ChaCha block with `rounds` rounds: a 64-bit block counter in words
// 12-13 and a zero 64-bit stream id in words 14-15 (rand_chacha's layout).
void chacha_block(const uint32_t key[8], uint64_t ctr, int rounds, uint32_t out[16]) {
  uint32_t st[16] = {0x61707865u, 0x3320646Eu, 0x79622D32u, 0x6B206574u};
  for (int i = 0; i < 8; ++i) st[4 + i] = key[i];
  st[12] = (uint32_t)ctr;
  st[13] = (uint32_t)(ctr >> 32);
  st[14] = 0;
  st[15] = 0;
  uint32_t x[16];
  memcpy(x, st, sizeof x);
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < rounds; r += 2) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + st[i];
}

uint32_t rng_next_u32(spec_rng* r) {
  if (r->pos >= 64) {
    for (int b = 0; b < 4; ++b) chacha_block(r->key, r->block + b, 12, r->buf + 16 * b);
    r->block += 4;
    r->pos = 0;
  }
  return r->buf[r->pos++];
}

// gen::<f32>(): the top 24 bits scaled by 2^-24 (exact in f32).
float rng_next_f32(spec_rng* r) { return (float)(rng_next_u32(r) >> 8) * (1.0f / 16777216.0f); }

void rng_peek_f32(const spec_rng* r, int n, float* out) {
  spec_rng c = *r;
  for (int i = 0; i < n; ++i) out[i] = rng_next_f32(&c);
}

}  // namespace

int spec_rng_create(uint64_t seed, spec_rng** out) {
  if (!out) return SPEC_ERR_INVALID;
  spec_rng* r = new (std::nothrow) spec_rng();
  if (!r) return SPEC_ERR_OOM;
  // rand_core 0.6 seed_from_u64: eight PCG32 outputs, little-endian.
  uint64_t state = seed;
  for (int i = 0; i < 8; ++i) {
    state = state * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27);
    const int rot = (int)(state >> 59);
    r->key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  *out = r;
  return SPEC_OK;
}

void spec_rng_free(spec_rng* r) { delete r; }

int spec_rng_next_f32(spec_rng* r, float* out, int n) {
  if (!r || (n > 0 && !out) || n < 0) return SPEC_ERR_INVALID;
  for (int i = 0; i < n; ++i) out[i] = rng_next_f32(r);
  return SPEC_OK;
}

int spec_sd_sampled_round(spec_model* target, spec_model* draft, int k, float temperature, spec_rng* rng, int budget,
                          uint32_t* commits_out, int* n_out, int* n_accepted) {
  if (!target || !draft || !rng || !commits_out || !n_out || k < 0 || k + 1 > kMaxRows) return SPEC_ERR_INVALID;
  if (budget < 1) return target->fail(SPEC_ERR_INVALID, "token budget must be >= 1");
  if (target->history.size() != draft->history.size())
    return target->fail(SPEC_ERR_INVALID, "target and draft histories differ in length");
  if (target->cfg.vocab != draft->cfg.vocab) return target->fail(SPEC_ERR_INVALID, "target and draft vocabularies differ");
  const int V = target->cfg.vocab;
  k = std::min(k, budget);
  const int pre = (int)target->history.size();
  uint32_t drafts[kMaxRows];
  auto draft_fail = [&](int rc) {
    if (draft != target) target->err = draft->err;
    return rc;
  };
  for (int i = 0; i < k; ++i) {
    // A zero-draft rejection round on the draft is its sampling step: one
    // forward of the pending token, softmax_t of the row (left in its logits
    // buffer as probabilities), a sample with the next draw.
    float u;
    rng_peek_f32(rng, 1, &u);
    uint32_t tok = 0;
    int nc = 0, used = 0;
    int rc = verify_rejection_core(draft, nullptr, 0, nullptr, temperature, &u, 1, 1, &tok, &nc, &used);
    if (rc == SPEC_OK && (nc != 1 || used != 1)) rc = draft->fail(SPEC_ERR_INVALID, "draft sampling step");
    if (rc != SPEC_OK) return draft_fail(rc);
    for (int j = 0; j < used; ++j) rng_next_f32(rng);
    // The row goes to the target's q buffer on the draft's stream: the next
    // draft step (same stream) overwrites the row only after the copy.
    DeviceGuard dg_(draft->device);
    cudaError_t e = cudaMemcpyAsync(target->rej_q + (size_t)i * V, draft->logits, (size_t)V * 4, cudaMemcpyDefault,
                                    draft->stream);
    if (e != cudaSuccess) return draft_fail(draft->fail(SPEC_ERR_CUDA, cuda_msg(e, "draft distribution copy")));
    rc = spec_observe(draft, &tok, 1);
    if (rc != SPEC_OK) return draft_fail(rc);
    drafts[i] = tok;
  }
  {
    DeviceGuard dg_(draft->device);
    const cudaError_t e = cudaStreamSynchronize(draft->stream);
    if (e != cudaSuccess) return draft_fail(draft->fail(SPEC_ERR_CUDA, cuda_msg(e, "draft distribution copy")));
  }
  float u[kMaxRows + 1];
  rng_peek_f32(rng, k + 1, u);
  uint32_t commits[kMaxRows];
  int n = 0, used = 0;
  int rc = verify_rejection_core(target, drafts, k, nullptr, temperature, u, k + 1, budget, commits, &n, &used);
  if (rc != SPEC_OK) return rc;
  for (int j = 0; j < used; ++j) rng_next_f32(rng);
  // Drafts accepted: a rejection or the bonus adds one commit beyond them; a
  // budget cut-off does not (then every draw was an accept test).
  const int n_acc = (used == n && n <= k) ? n : n - 1;
  const int acc = std::min(n, k);
  rc = spec_rollback_to(target, pre + acc);
  if (rc == SPEC_OK && n > acc) rc = spec_observe(target, commits + acc, n - acc);
  if (rc == SPEC_OK) rc = spec_rollback_to(draft, pre + acc);
  if (rc == SPEC_OK && n > acc) rc = spec_observe(draft, commits + acc, n - acc);
  if (rc != SPEC_OK) return rc;
  for (int i = 0; i < n; ++i) commits_out[i] = commits[i];
  *n_out = n;
  if (n_accepted) *n_accepted = n_acc;
  return SPEC_OK;
}

// spec_verify_tree_greedy; with `hidden` the tree forward also leaves every
// node's final hidden row in m->hidden_out (device).
int verify_tree_greedy_core(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, int32_t* best_path,
                            int* path_len, uint32_t* bonus, bool hidden) {
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  int rc = check_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  if (tokens[0] != m->history.back()) return m->fail(SPEC_ERR_INVALID, "tree root must equal last committed token");
  // The root is the last committed token, at position history - 1 (its KV
  // row may still be pending after a lazy observe; the tree forward writes it).
  const int pre = m->cache_len;
  const int prefix = (int)m->history.size() - 1;
  if (prefix > pre) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  rc = tree_forward(m, tokens, parents, n, prefix, hidden ? (F_LOGITS | F_HIDDEN) : F_LOGITS);
  if (rc == SPEC_OK) {
    cudaError_t e = launch_row_argmax(m->logits, n, m->cfg.vocab, m->argmax_dev, nullptr,
                                      m->argmax_slots, m->argmax_counters, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(m->argmax_host, m->argmax_dev, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "argmax"));
  }
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) return rc;
  m->cache_len = prefix + n;
  // eagle.rs:618-661: walk every root-to-leaf path (leaves in index order),
  // count leading matches, keep the first longest.
  std::vector<char> is_leaf(n, 1);
  for (int i = 1; i < n; ++i) is_leaf[parents[i]] = 0;
  std::vector<int> best = {0};
  for (int leaf = 0; leaf < n; ++leaf) {
    if (!is_leaf[leaf]) continue;
    std::vector<int> chain;
    for (int cur = leaf;; cur = parents[cur]) {
      chain.push_back(cur);
      if (cur == 0) break;
    }
    std::reverse(chain.begin(), chain.end());
    int accepted = 0;
    for (size_t w = 0; w + 1 < chain.size(); ++w) {
      if ((uint32_t)m->argmax_host[chain[w]] == tokens[chain[w + 1]]) ++accepted;
      else break;
    }
    if (accepted + 1 > (int)best.size()) best.assign(chain.begin(), chain.begin() + accepted + 1);
  }
  for (size_t i = 0; i < best.size(); ++i) best_path[i] = best[i];
  *path_len = (int)best.size();
  *bonus = (uint32_t)m->argmax_host[best.back()];
  return SPEC_OK;
}

int spec_verify_tree_greedy(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                            int32_t* best_path, int* path_len, uint32_t* bonus) {
  if (!m || !tokens || !parents || !best_path || !path_len || !bonus) return SPEC_ERR_INVALID;
  if (n <= kMaxRows) return verify_tree_greedy_core(m, tokens, parents, n, best_path, path_len, bonus, false);
  // Over kMaxRows nodes: the chunk forwards' argmaxes, the same walk.
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  std::vector<int32_t> am(n);
  int rc = big_tree_keep_kv(m, tokens, parents, n, nullptr, nullptr, am.data());
  if (rc != SPEC_OK) return rc;
  std::vector<char> is_leaf(n, 1);
  for (int i = 1; i < n; ++i) is_leaf[parents[i]] = 0;
  std::vector<int> best = {0}, chain;
  for (int leaf = 0; leaf < n; ++leaf) {
    if (!is_leaf[leaf]) continue;
    chain.clear();
    for (int cur = leaf;; cur = parents[cur]) {
      chain.push_back(cur);
      if (cur == 0) break;
    }
    std::reverse(chain.begin(), chain.end());
    int accepted = 0;
    for (size_t w = 0; w + 1 < chain.size(); ++w) {
      if ((uint32_t)am[chain[w]] == tokens[chain[w + 1]]) ++accepted;
      else break;
    }
    if (accepted + 1 > (int)best.size()) best.assign(chain.begin(), chain.begin() + accepted + 1);
  }
  for (size_t i = 0; i < best.size(); ++i) best_path[i] = best[i];
  *path_len = (int)best.size();
  *bonus = (uint32_t)am[best.back()];
  return SPEC_OK;
}

// Medusa's typical acceptance (medusa.rs:290-326 with Acceptance::Typical,
// :391-445) over one tree forward with the KV kept: the per-node pass/fail
// flags come from the device (typical_accept_kernel, the reference's f32
// operations in its order), the path walk and the argmax bonus are those of
// spec_verify_tree_greedy.
// With `hidden` the tree forward also leaves every node's final hidden row in
// m->hidden_out (device).
int verify_tree_typical_core(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float epsilon,
                             float delta, int32_t* best_path, int* path_len, uint32_t* bonus, bool hidden) {
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  int rc = check_tree(m, tokens, parents, n);
  if (rc != SPEC_OK) return rc;
  if (tokens[0] != m->history.back()) return m->fail(SPEC_ERR_INVALID, "tree root must equal last committed token");
  const int pre = m->cache_len;
  const int prefix = (int)m->history.size() - 1;
  if (prefix > pre) return m->fail(SPEC_ERR_CACHE_ROLLBACK, "truncate beyond cache length");
  TypicalTree tt;
  tt.n = n;
  tt.epsilon = epsilon;
  tt.delta = delta;
  for (int i = 0; i < n; ++i) {
    tt.tok[i] = tokens[i];
    tt.par[i] = i ? parents[i] : 0;
  }
  int* flags_dev = m->rej_out_dev + 4;  // kMaxRows ints
  int* flags_host = m->rej_out_host + 4;
  rc = tree_forward(m, tokens, parents, n, prefix, hidden ? (F_LOGITS | F_HIDDEN) : F_LOGITS);
  if (rc == SPEC_OK) {
    cudaError_t e = launch_row_argmax(m->logits, n, m->cfg.vocab, m->argmax_dev, nullptr, m->argmax_slots,
                                      m->argmax_counters, m->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(flags_dev, 0, (size_t)n * 4, m->stream);
    if (e == cudaSuccess) e = launch_typical_accept(m->logits, m->cfg.vocab, tt, flags_dev, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(m->argmax_host, m->argmax_dev, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(flags_host, flags_dev, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = m->fail(SPEC_ERR_CUDA, cuda_msg(e, "typical acceptance"));
  }
  if (rc == SPEC_OK) rc = finish(m);
  if (rc != SPEC_OK) return rc;
  m->cache_len = prefix + n;
  std::vector<char> is_leaf(n, 1);
  for (int i = 1; i < n; ++i) is_leaf[parents[i]] = 0;
  std::vector<int> best = {0};
  for (int leaf = 0; leaf < n; ++leaf) {
    if (!is_leaf[leaf]) continue;
    std::vector<int> chain;
    for (int cur = leaf;; cur = parents[cur]) {
      chain.push_back(cur);
      if (cur == 0) break;
    }
    std::reverse(chain.begin(), chain.end());
    int accepted = 0;
    for (size_t w = 0; w + 1 < chain.size(); ++w) {
      if (flags_host[chain[w + 1]]) ++accepted;
      else break;
    }
    if (accepted + 1 > (int)best.size()) best.assign(chain.begin(), chain.begin() + accepted + 1);
  }
  for (size_t i = 0; i < best.size(); ++i) best_path[i] = best[i];
  *path_len = (int)best.size();
  *bonus = (uint32_t)m->argmax_host[best.back()];
  return SPEC_OK;
}

// Over kMaxRows nodes: after each chunk's forward, the children of the
// chunk's primary nodes are decided against their parents' rows, up to
// kMaxRows - 1 at a time (kernel slots 1.., parent = the parent's row in the
// chunk, -1 in unused slots); then the walk of the small-tree path.
static int big_verify_tree_typical(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n,
                                   float epsilon, float delta, int32_t* best_path, int* path_len, uint32_t* bonus) {
  std::vector<int32_t> am(n);
  std::vector<char> pass(n, 0);
  std::vector<std::vector<int>> kids(n);
  for (int i = 1; i < n; ++i)
    if (parents[i] >= 0 && parents[i] < i) kids[parents[i]].push_back(i);
  int* flags_dev = m->rej_out_dev + 4;  // kMaxRows ints
  int* flags_host = m->rej_out_host + 4;
  auto decide = [&](const TreeChunk& c, const std::vector<int>& local) -> int {
    std::vector<std::pair<int, int>> q;  // (row in the chunk, child node)
    for (int p : c.primary)
      for (int ch : kids[p]) q.push_back({local[p], ch});
    const int cn = (int)c.nodes.size();
    for (size_t b = 0; b < q.size(); b += kMaxRows - 1) {
      const int nq = (int)std::min<size_t>(kMaxRows - 1, q.size() - b);
      TypicalTree tt;
      tt.n = std::max(cn, nq + 1);
      tt.epsilon = epsilon;
      tt.delta = delta;
      for (int i = 0; i < tt.n; ++i) {
        tt.tok[i] = 0;
        tt.par[i] = -1;
      }
      for (int j = 0; j < nq; ++j) {
        tt.par[j + 1] = q[b + j].first;
        tt.tok[j + 1] = tokens[q[b + j].second];
      }
      cudaError_t e = cudaMemsetAsync(flags_dev, 0, (size_t)tt.n * 4, m->stream);
      if (e == cudaSuccess) e = launch_typical_accept(m->logits, m->cfg.vocab, tt, flags_dev, m->stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(flags_host, flags_dev, (size_t)tt.n * 4, cudaMemcpyDeviceToHost, m->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
      if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "typical acceptance"));
      for (int j = 0; j < nq; ++j) pass[q[b + j].second] = flags_host[j + 1] != 0;
    }
    return SPEC_OK;
  };
  int rc = big_tree_keep_kv(m, tokens, parents, n, nullptr, nullptr, am.data(), decide);
  if (rc != SPEC_OK) return rc;
  std::vector<char> is_leaf(n, 1);
  for (int i = 1; i < n; ++i) is_leaf[parents[i]] = 0;
  std::vector<int> best = {0}, chain;
  for (int leaf = 0; leaf < n; ++leaf) {
    if (!is_leaf[leaf]) continue;
    chain.clear();
    for (int cur = leaf;; cur = parents[cur]) {
      chain.push_back(cur);
      if (cur == 0) break;
    }
    std::reverse(chain.begin(), chain.end());
    int accepted = 0;
    for (size_t w = 0; w + 1 < chain.size(); ++w) {
      if (pass[chain[w + 1]]) ++accepted;
      else break;
    }
    if (accepted + 1 > (int)best.size()) best.assign(chain.begin(), chain.begin() + accepted + 1);
  }
  for (size_t i = 0; i < best.size(); ++i) best_path[i] = best[i];
  *path_len = (int)best.size();
  *bonus = (uint32_t)am[best.back()];
  return SPEC_OK;
}

int spec_verify_tree_typical(spec_model* m, const uint32_t* tokens, const int32_t* parents, int n, float epsilon,
                             float delta, int32_t* best_path, int* path_len, uint32_t* bonus) {
  if (!m || !tokens || !parents || !best_path || !path_len || !bonus) return SPEC_ERR_INVALID;
  if (n <= kMaxRows)
    return verify_tree_typical_core(m, tokens, parents, n, epsilon, delta, best_path, path_len, bonus, false);
  DeviceGuard dg_(m->device);
  m->last_valid = false;
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "tree_logits with empty history");
  return big_verify_tree_typical(m, tokens, parents, n, epsilon, delta, best_path, path_len, bonus);
}

// The EAGLE-2 round tree (eagle.rs:584-593): the Cartesian product of the
// draft steps' top-k (medusa.rs:172-189: BFS layers, every candidate of step
// d under every node of layer d, parents in layer order), pruned to at most
// max_nodes by path log-prob (eagle.rs:763-843).  In that tree node p of
// layer D (0-based position) has parent p / k of layer D-1 and candidate
// p % k of step D-1, so nothing is materialised but the scores.  The score
// is the f32 sum of the candidates' log-probs deepest step first (:800-812);
// the first max_nodes - 1 of the stable descending sort (:815) are the
// max_nodes - 1 largest under (score desc, index asc); their ancestors are
// added (:822-827) and the kept nodes keep their BFS order, which is the
// depth order (:829-842).
int spec_eagle_build_tree(uint32_t root, const int32_t* ids, const float* logprobs, int depth, int k, int max_nodes,
                          uint32_t* tokens_out, int32_t* parents_out, int cap, int* n_out) {
  if (!ids || !tokens_out || !parents_out || !n_out || depth < 0 || k < 1 || cap < 1 ||
      (max_nodes > 0 && !logprobs))
    return SPEC_ERR_INVALID;
  std::vector<int64_t> start(depth + 2, 0);  // first index of each layer
  int64_t width = 1;
  for (int d = 0; d <= depth; ++d) {
    start[d + 1] = start[d] + width;
    if (start[d + 1] > (int64_t)1 << 26) {
      set_thread_error("spec_eagle_build_tree: the Cartesian tree exceeds 2^26 nodes");
      return SPEC_ERR_UNSUPPORTED;
    }
    width *= k;
  }
  const int64_t N = start[depth + 1];
  auto layer_of = [&](int64_t i) {
    int d = 0;
    while (start[d + 1] <= i) ++d;
    return d;
  };
  std::vector<char> keep;
  if (max_nodes > 0 && N > max_nodes) {
    std::vector<float> score((size_t)(N - 1));
    for (int D = 1; D <= depth; ++D)
      for (int64_t p = 0; p < start[D + 1] - start[D]; ++p) {
        float sc = 0.f;
        int64_t q = p;
        for (int d = D - 1; d >= 0; --d) {
          sc += logprobs[(size_t)d * k + (q % k)];
          q /= k;
        }
        score[(size_t)(start[D] + p - 1)] = sc;
      }
    std::vector<int32_t> order((size_t)(N - 1));
    std::iota(order.begin(), order.end(), 1);
    const int64_t want = std::min<int64_t>(max_nodes - 1, N - 1);
    auto before = [&](int32_t a, int32_t b) {
      const float sa = score[(size_t)a - 1], sb = score[(size_t)b - 1];
      return sa > sb || (!(sb > sa) && a < b);
    };
    std::nth_element(order.begin(), order.begin() + want, order.end(), before);
    keep.assign((size_t)N, 0);
    keep[0] = 1;
    for (int64_t j = 0; j < want; ++j) keep[(size_t)order[(size_t)j]] = 1;
    for (int64_t i = N - 1; i >= 1; --i)
      if (keep[(size_t)i]) {
        const int D = layer_of(i);
        keep[(size_t)(start[D - 1] + (i - start[D]) / k)] = 1;
      }
  } else {
    keep.assign((size_t)N, 1);
  }
  std::vector<int64_t> new_index((size_t)N, -1);
  int n = 0;
  for (int64_t i = 0; i < N; ++i) {
    if (!keep[(size_t)i]) continue;
    if (n >= cap) {
      set_thread_error("spec_eagle_build_tree: the tree has more nodes than the output capacity");
      return SPEC_ERR_UNSUPPORTED;
    }
    new_index[(size_t)i] = n;
    if (i == 0) {
      tokens_out[0] = root;
      parents_out[0] = 0;
    } else {
      const int D = layer_of(i);
      const int64_t p = i - start[D];
      tokens_out[n] = (uint32_t)ids[(size_t)(D - 1) * k + (p % k)];
      parents_out[n] = (int32_t)new_index[(size_t)(start[D - 1] + p / k)];
    }
    ++n;
  }
  *n_out = n;
  return SPEC_OK;
}

int spec_eagle_round(spec_model* m, const float* hidden, int depth, int top_k, int max_tree_nodes, int strict_root,
                     const uint32_t* eos_ids, int n_eos, uint32_t* commits_out, int* n_out, float* hidden_out,
                     int* stop) {
  if (!m || !hidden || !commits_out || !n_out || !hidden_out || !stop || depth < 1 || top_k < 1 || n_eos < 0 ||
      (n_eos > 0 && !eos_ids))
    return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "EAGLE round with empty history");
  const uint32_t root = m->history.back();
  // 1-2. Draft loop from the target's hidden row at the history length.
  std::vector<int32_t> ids((size_t)depth * top_k);
  std::vector<float> lps((size_t)depth * top_k);
  int rc = spec_eagle_draft(m, hidden, root, (int)m->history.size(), depth, top_k, ids.data(), lps.data());
  if (rc != SPEC_OK) return rc;
  // 3. The tree.  Over kMaxRows nodes the tree forward runs as
  // ancestor-closed chunks (spec_verify_tree_greedy) and the bonus is always
  // observed (no per-node hidden rows are kept).
  constexpr int kMaxEagleNodes = 1 << 14;
  std::vector<uint32_t> tok(kMaxEagleNodes);
  std::vector<int32_t> par(kMaxEagleNodes);
  int n = 0;
  rc = spec_eagle_build_tree(root, ids.data(), lps.data(), depth, top_k, max_tree_nodes, tok.data(), par.data(),
                             kMaxEagleNodes, &n);
  if (rc != SPEC_OK) return m->fail(rc, g_load_error.empty() ? "EAGLE tree" : g_load_error);
  const bool small = n <= kMaxRows;
  // 4-6. Tree forward keeping KV, greedy walk, bonus (per-node hidden kept).
  std::vector<int32_t> best((size_t)n + 1);
  int len = 0;
  uint32_t bonus = 0;
  rc = small ? verify_tree_greedy_core(m, tok.data(), par.data(), n, best.data(), &len, &bonus, true)
             : spec_verify_tree_greedy(m, tok.data(), par.data(), n, best.data(), &len, &bonus);
  if (rc != SPEC_OK) return rc;
  auto is_eos = [&](uint32_t t) {
    for (int i = 0; i < n_eos; ++i)
      if (eos_ids[i] == t) return true;
    return false;
  };
  int nc = 0;
  for (int i = 1; i < len; ++i) commits_out[nc++] = tok[best[i]];
  commits_out[nc++] = bonus;
  int eos_at = -1;
  for (int i = 0; i < nc; ++i)
    if (is_eos(commits_out[i])) {
      eos_at = i;
      break;
    }
  if (eos_at >= 0) nc = eos_at + 1;
  *n_out = nc;
  *stop = eos_at >= 0 ? 1 : 0;
  // 7. Commit the accepted path.
  if (eos_at >= 0 && eos_at < len - 1) {
    // An EOS on the accepted path: keep the root and the path up to it.
    return spec_commit_tree_path(m, tok.data(), par.data(), n, best.data(), eos_at + 2);
  }
  const int deepest = best[len - 1];
  int bn = -1;
  if (!strict_root && small)
    for (int i = 1; i < n; ++i)
      if (par[i] == deepest && tok[i] == bonus) {
        bn = i;
        break;
      }
  if (bn >= 0) {
    // The bonus is a child of the deepest accepted node: its KV row is in
    // the cache already and its hidden row comes from the tree forward.
    const cudaError_t e = cudaMemcpy(hidden_out, m->hidden_out + (size_t)bn * m->cfg.hidden,
                                     (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "tree hidden row"));
    best[len++] = bn;
    return spec_commit_tree_path(m, tok.data(), par.data(), n, best.data(), len);
  }
  rc = spec_commit_tree_path(m, tok.data(), par.data(), n, best.data(), len);
  if (rc == SPEC_OK) rc = spec_observe_returning_last_hidden(m, &bonus, 1, hidden_out);
  return rc;
}

// One Medusa round: the body of run_medusa_real's loop (medusa.rs:761-810).
// The reference's tree_logits restores the state and observe(committed)
// recomputes the accepted rows; here the tree forward keeps its KV rows and
// the accepted path is committed in place (spec_commit_tree_path), then the
// bonus is observed, which leaves the same history and KV rows.
int spec_medusa_round(spec_model* m, const float* hidden, int top_k, int topology, int acceptance, float epsilon,
                      float delta, int budget, uint32_t* commits_out, int* n_out, float* hidden_out) {
  if (!m || !hidden || !commits_out || !n_out || !hidden_out || top_k < 1 || (topology != 0 && topology != 1) ||
      (acceptance != 0 && acceptance != 1))
    return SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return m->fail(SPEC_ERR_INVALID, "Medusa requires non-empty prompt");
  if (budget < 1) return m->fail(SPEC_ERR_INVALID, "token budget must be >= 1");
  MedusaHeads* h = m->medusa.get();
  if (!h) return m->fail(SPEC_ERR_INVALID, "no Medusa heads attached (spec_medusa_attach)");
  const int nh = h->n_heads;
  const uint32_t root = m->history.back();
  // 1. Per-head top-k from the target's last hidden row (:766-768).
  std::vector<int32_t> ids((size_t)nh * top_k);
  int rc = spec_medusa_topk(m, hidden, top_k, ids.data(), nullptr);
  if (rc != SPEC_OK) return rc;
  // 2. The tree (:771): a chain of each head's top-1 (:167-170), or BFS
  // layers with every candidate of head d under every node of layer d
  // (:172-189).  Over kMaxRows nodes it runs as ancestor-closed chunks.
  constexpr int64_t kMaxMedusaNodes = 1 << 14;
  int64_t total = 1;
  if (topology == 0) {
    total = 1 + nh;
  } else {
    int64_t width = 1;
    for (int d = 0; d < nh; ++d) {
      width *= top_k;
      total += width;
      if (total > kMaxMedusaNodes) break;
    }
  }
  if (total > kMaxMedusaNodes) return m->fail(SPEC_ERR_UNSUPPORTED, "Medusa tree larger than 16384 nodes");
  std::vector<uint32_t> tok((size_t)total);
  std::vector<int32_t> par((size_t)total);
  int n = 1;
  tok[0] = root;
  par[0] = 0;
  if (topology == 0) {
    for (int d = 0; d < nh; ++d) {
      tok[n] = (uint32_t)ids[(size_t)d * top_k];
      par[n] = n - 1;
      ++n;
    }
  } else {
    int lo = 0, hi = 1;  // the previous layer's node range
    for (int d = 0; d < nh; ++d) {
      const int start = n;
      for (int p = lo; p < hi; ++p)
        for (int c = 0; c < top_k; ++c) {
          tok[n] = (uint32_t)ids[(size_t)d * top_k + c];
          par[n] = p;
          ++n;
        }
      lo = start;
      hi = n;
    }
  }
  // 3-4. Tree forward (KV kept; per-node hidden rows too up to kMaxRows
  // nodes) and the walk.
  const bool small = n <= kMaxRows;
  std::vector<int32_t> best((size_t)n);
  int len = 0;
  uint32_t bonus = 0;
  if (small)
    rc = acceptance == 0 ? verify_tree_greedy_core(m, tok.data(), par.data(), n, best.data(), &len, &bonus, true)
                         : verify_tree_typical_core(m, tok.data(), par.data(), n, epsilon, delta, best.data(), &len,
                                                    &bonus, true);
  else
    rc = acceptance == 0 ? spec_verify_tree_greedy(m, tok.data(), par.data(), n, best.data(), &len, &bonus)
                         : spec_verify_tree_typical(m, tok.data(), par.data(), n, epsilon, delta, best.data(), &len,
                                                    &bonus);
  if (rc != SPEC_OK) return rc;
  // 5. Commit, with the bonus while the budget allows (:786-800).
  int nc = 0;
  for (int i = 1; i < len; ++i) commits_out[nc++] = tok[best[i]];
  const bool with_bonus = nc < budget;
  if (with_bonus) commits_out[nc++] = bonus;
  *n_out = nc;
  if (!with_bonus) {
    if (small) {
      const cudaError_t e = cudaMemcpy(hidden_out, m->hidden_out + (size_t)best[len - 1] * m->cfg.hidden,
                                       (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "tree hidden row"));
    }
    rc = spec_commit_tree_path(m, tok.data(), par.data(), n, best.data(), len);
    if (rc == SPEC_OK && !small) rc = spec_last_hidden_state(m, hidden_out);
    return rc;
  }
  rc = spec_commit_tree_path(m, tok.data(), par.data(), n, best.data(), len);
  if (rc == SPEC_OK) rc = spec_observe_returning_last_hidden(m, &bonus, 1, hidden_out);
  return rc;
}

float spec_last_forward_ms(const spec_model* m) { return m ? m->last_ms : 0.f; }

}  // extern "C"

struct spec_qweight {
  std::unique_ptr<spec_model> ctx;
  Mat mat;
  uint32_t* frag = nullptr;
  float* x16 = nullptr;
  float* x32 = nullptr;
  float* y = nullptr;
  void* flush = nullptr;
  size_t flush_bytes = 0;
  int last_M = 0;
  FwdOp* op_dev = nullptr;  // descriptor of the last launched matmul
  int* op_done = nullptr;
  int op_M = 0;  // the slot's descriptor is a function of (M, output) only
  float* op_out = nullptr;
};

extern "C" {

int spec_qweight_upload(int ggml_type, const void* gguf_blocks, int n_rows, int k_cols, int device,
                        spec_qweight** out) {
  if (!out || !gguf_blocks || n_rows <= 0 || k_cols <= 0) return SPEC_ERR_INVALID;
  *out = nullptr;
  std::unique_ptr<spec_qweight> w(new (std::nothrow) spec_qweight());
  if (!w) return SPEC_ERR_OOM;
  w->ctx.reset(new spec_model());
  spec_model* m = w->ctx.get();
  spec_load_opts o = {};
  o.device = device;
  DeviceGuard dg_(device);
  int rc = init_device(m, &o);
  if (rc != SPEC_OK) {
    g_load_error = m->err;
    return rc;
  }
  Part p;
  p.src = static_cast<const uint8_t*>(gguf_blocks);
  p.on_device = false;
  p.fmt = ggml_type;
  p.rows = n_rows;
  if (fmt_tile_bytes(ggml_type) == 0 || k_cols % fmt_kt(ggml_type) || n_rows % kGroupRows) {
    g_load_error = "unsupported format or shape (rows must be a multiple of 128, K of the tile width)";
    return SPEC_ERR_UNSUPPORTED;
  }
  rc = build_mat(m, {p}, k_cols, false, w->mat);
  cudaError_t e = cudaSuccess;
  const int groups = w->mat.seg[0].groups;
  if (rc == SPEC_OK) e = m->dalloc(&w->frag, (size_t)k_cols * kMaxRows * 2);
  if (e == cudaSuccess && rc == SPEC_OK) e = m->dalloc(&w->x16, (size_t)(k_cols / 16) * kMaxRows * 4);
  if (e == cudaSuccess && rc == SPEC_OK) e = m->dalloc(&w->x32, (size_t)(k_cols / 32) * kMaxRows * 4);
  if (e == cudaSuccess && rc == SPEC_OK) e = m->dalloc(&w->y, (size_t)n_rows * kMaxRows * 4);
  if (e == cudaSuccess && rc == SPEC_OK)
    e = m->dalloc(&m->gemv_part, (size_t)partial_slots(w->mat) * kGroupRows * kMaxRows * 4);
  if (e == cudaSuccess && rc == SPEC_OK) e = m->dalloc(&m->counters, (size_t)groups * 4);
  if (e == cudaSuccess && rc == SPEC_OK) e = m->dalloc(&m->err_dev, 16);
  if (e == cudaSuccess && rc == SPEC_OK) e = cudaStreamSynchronize(m->stream);
  if (rc == SPEC_OK && e != cudaSuccess) rc = m->fail(SPEC_ERR_OOM, cuda_msg(e, "qweight buffers"));
  if (rc != SPEC_OK) {
    g_load_error = m->err;
    return rc;
  }
  *out = w.release();
  return SPEC_OK;
}

void spec_qweight_free(spec_qweight* w) {
  if (!w) return;
  if (w->flush) {
    DeviceGuard dg_(w->ctx->device);
    cudaFree(w->flush);
  }
  delete w;
}

int64_t spec_qweight_bytes(const spec_qweight* w) { return w ? w->mat.bytes : 0; }

static int qmatmul_enqueue(spec_qweight* w, int M, float* y_dev, cudaStream_t s) {
  spec_model* m = w->ctx.get();
  QmvParams p = base_params(m, w->mat, M);
  p.act_bf16 = w->mat.seg[0].fmt == WF_BF16 ? 1 : 0;
  p.xfrag = w->frag;
  p.xsum16 = w->x16;
  p.xsum32 = w->x32;
  p.epi = EPI_STORE;
  p.out = y_dev;
  p.ld_out = w->mat.N;
  cudaError_t e = cudaSuccess;
  if (!w->op_dev) {
    e = m->dalloc(&w->op_dev, sizeof(FwdOp));
    if (e == cudaSuccess) e = m->dalloc(&w->op_done, 16);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "qmatmul op slot"));
  }
  if (w->op_M != M || w->op_out != y_dev) {
    FwdOp op{};
    op.q = p;
    op.dep = -1;
    // New descriptor: the slot may still feed a launch in flight (on any
    // stream), so drain the device first.  Happens once per (M, output).
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = m->upload(w->op_dev, &op, sizeof(FwdOp));
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "qmatmul op upload"));
    w->op_M = M;
    w->op_out = y_dev;
  }
  if (!m->fmt_set) m->fmt_set = fwd_fmt_set_for(m->fmt_bits);
  FwdParams fp;
  fp.ops = w->op_dev;
  fp.n_ops = 1;
  fp.done = w->op_done;  // nothing waits on it: one op per launch
  fp.err = m->err_dev;
  fp.l2_ahead = m->l2_ahead;
  e = launch_fwd(fp, m->fmt_set, M, s, false);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "qmatmul launch"));
  return SPEC_OK;
}

}  // extern "C"

namespace specb200 {

bool qweight_launch_desc(spec_qweight* w, int M, float* y_dev, QmatmulLaunch* out) {
  if (!w || !out) return false;
  spec_model* m = w->ctx.get();
  QmvParams p = base_params(m, w->mat, M);
  p.part = nullptr;
  p.counters = nullptr;
  p.act_bf16 = w->mat.seg[0].fmt == WF_BF16 ? 1 : 0;
  p.epi = EPI_STORE;
  p.out = y_dev;
  p.ld_out = w->mat.N;
  out->p = p;
  out->fmt_set = m->fmt_set ? m->fmt_set : fwd_fmt_set_for(m->fmt_bits);
  out->device = m->device;
  out->l2_ahead = m->l2_ahead;
  out->stream = m->stream;
  return true;
}

void set_thread_error(const char* msg) { g_load_error = msg; }

int take_device_error(unsigned* err_dev, cudaStream_t s, char* msg, size_t cap) {
  unsigned h[4] = {0u, 0u, 0u, 0u};
  cudaError_t e = cudaMemcpyAsync(h, err_dev, sizeof h, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    snprintf(msg, cap, "reading the device error word: %s", cudaGetErrorString(e));
    return SPEC_ERR_CUDA;
  }
  if (!h[0]) return SPEC_OK;
  e = cudaMemsetAsync(err_dev, 0, sizeof h, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (h[0] & DEV_ERR_MBAR_TIMEOUT) {
    snprintf(msg, cap,
             "a device wait gave up (mbarrier timeout): site %u op %u cta %u, stage/pos %u (0x%x), counter %d; "
             "the output is incomplete",
             h[1] & 0xffu, (h[1] >> 8) & 0xffu, h[1] >> 16, h[2], h[2], (int)h[3]);
    return SPEC_ERR_TIMEOUT;
  }
  snprintf(msg, cap, "a kernel rejected an argument (device error bits 0x%x)", h[0]);
  return SPEC_ERR_INVALID;
}

}  // namespace specb200

extern "C" {

static int qmatmul_call(spec_qweight* w, const float* x_dev, int M, float* y_dev, void* stream) {
  spec_model* m = w->ctx.get();
  DeviceGuard dg(m->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  const int nt = nt_for_rows(M);
  cudaError_t e = launch_make_operand(x_dev, M, w->mat.K, nt, w->frag, w->x16, w->x32,
                                      w->mat.seg[0].fmt == WF_BF16 ? 1 : 0, s);
  if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "operand"));
  w->last_M = M;
  int rc = qmatmul_enqueue(w, M, y_dev, s);
  if (rc != SPEC_OK) return rc;
  if (!stream) {
    // Synchronous call: a bounded wait that gave up inside the kernel left
    // y incomplete; report it (and clear the word) instead of SPEC_OK.
    char msg[256];
    rc = take_device_error(m->err_dev, s, msg, sizeof msg);
    if (rc != SPEC_OK) return m->fail(rc, msg);
  }
  return SPEC_OK;
}

int spec_qmatmul(spec_qweight* w, const float* x_dev, int M, float* y_dev, void* stream) {
  if (!w || !x_dev || !y_dev || M < 1 || M > kMaxRows) {
    g_load_error = "spec_qmatmul: null argument or M outside [1, 64]";
    return SPEC_ERR_INVALID;
  }
  const int rc = qmatmul_call(w, x_dev, M, y_dev, stream);
  // Weight calls report through spec_last_error(NULL) (this thread).
  if (rc != SPEC_OK) g_load_error = "spec_qmatmul: " + w->ctx->err;
  return rc;
}

int spec_qmatmul_time(spec_qweight* w, int M, int iters, int flush_l2, float* avg_ms) {
  if (!w || !avg_ms || iters < 1 || M != w->last_M) return SPEC_ERR_INVALID;
  spec_model* m = w->ctx.get();
  DeviceGuard dg_(m->device);
  cudaError_t e = cudaSuccess;
  if (flush_l2 && !w->flush) {
    w->flush_bytes = (size_t)512 << 20;
    e = cudaMalloc(&w->flush, w->flush_bytes);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_OOM, cuda_msg(e, "flush buffer"));
  }
  if (!m->ev0) {
    e = cudaEventCreate(&m->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&m->ev1);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "events"));
  }
  {  // untimed launch: uploads the descriptor for the timing output buffer
    int rc = qmatmul_enqueue(w, M, w->y, m->stream);
    if (rc != SPEC_OK) return rc;
  }
  double total = 0.0;
  for (int i = 0; i < iters; ++i) {
    if (flush_l2) e = cudaMemsetAsync(w->flush, i & 0xff, w->flush_bytes, m->stream);
    if (e == cudaSuccess) e = cudaEventRecord(m->ev0, m->stream);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "time"));
    int rc = qmatmul_enqueue(w, M, w->y, m->stream);
    if (rc != SPEC_OK) return rc;
    e = cudaEventRecord(m->ev1, m->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(m->ev1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, m->ev0, m->ev1);
    if (e != cudaSuccess) return m->fail(SPEC_ERR_CUDA, cuda_msg(e, "time"));
    total += ms;
  }
  *avg_ms = (float)(total / iters);
  return SPEC_OK;
}

void* spec_cuda_stream(const spec_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

int spec_profile_forward(spec_model* m, const uint32_t* drafts, int k, float* ms_out, int* kind_out,
                         int64_t* bytes_out, int cap) {
  if (!m || k < 0 || (k > 0 && !drafts) || !ms_out || !kind_out || !bytes_out) return -SPEC_ERR_INVALID;
  DeviceGuard dg_(m->device);
  if (m->history.empty()) return -m->fail(SPEC_ERR_INVALID, "profile with empty history");
  const int target = (int)m->history.size() - 1;
  if (target > m->cache_len || target + k + 1 > m->t_max) return -m->fail(SPEC_ERR_INVALID, "bad cache state");
  std::vector<uint32_t> combined(k + 1);
  combined[0] = m->history.back();
  if (k) memcpy(combined.data() + 1, drafts, (size_t)k * 4);
  fill_step_causal(m, combined.data(), k + 1, target);
  if (m->tp_size > 1 && !m->tp_connected)
    return -m->fail(SPEC_ERR_INVALID, "tensor-parallel handle used before spec_tp_connect");
  begin_step(m, F_LOGITS);
  ProfRec pr;
  cudaError_t e = enqueue_forward(m, k + 1, F_LOGITS, nullptr, &pr);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  int n = 0;
  if (e == cudaSuccess) {
    for (size_t i = 0; i + 1 < pr.ev.size() && n < cap; ++i, ++n) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, pr.ev[i], pr.ev[i + 1]);
      ms_out[n] = ms;
      kind_out[n] = pr.kind[i];
      bytes_out[n] = pr.bytes[i];
    }
  }
  for (cudaEvent_t ev : pr.ev) cudaEventDestroy(ev);
  // The forward rewrote KV rows [target, target + k]; the decoder's logical
  // state (history, cache_len) is unchanged and later forwards overwrite them.
  m->last_valid = false;
  if (e != cudaSuccess) return -m->fail(SPEC_ERR_CUDA, cuda_msg(e, "profile"));
  return n;
}

int spec_kernels_per_forward(const spec_model* m, int rows) {
  if (!m) return 0;
  // embed + layer-0 qkv (+ its attention) + per layer one multi-op launch
  // (o / gate-up / down / next qkv and attention, or the LM head); with
  // attention as its own kernels, a split and a combine launch per layer.
  const bool fused = rows >= 1 && rows <= kMaxRows && attn_fused(m, rows);
  return 2 + (fused ? 1 : 3) * m->cfg.n_layers;
}

int64_t spec_weight_bytes(const spec_model* m) { return m ? m->weight_bytes : 0; }

}  // extern "C"
