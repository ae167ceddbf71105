// Host-side model runtime of the verify-step backend (internal header).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "kernels.cuh"

namespace specb200 {

struct ModelCfg {
  int arch = 0;  // 0 llama, 1 qwen2
  int n_layers = 0, hidden = 0, n_heads = 0, n_kv = 0, head_dim = 0, ffn = 0, vocab = 0, ctx_len = 0;
  float eps = 1e-5f, rope_theta = 10000.f;
  bool rope_interleaved = true;  // GGUF Llama: rope_i; Qwen2 and BF16 Llama: rotate-half
  bool bf16 = false;             // BF16 weights: bf16 activations and KV
  bool has_bias = false;         // Qwen2 q/k/v biases
  bool rope_scaled = false;      // Llama-3.1 frequency scaling
  float rs_factor = 8.f, rs_low = 1.f, rs_high = 4.f;
  int rs_orig = 8192;
  bool rope_tables_bf16 = false; // BF16 model: cos/sin rounded to bf16
};

struct Mat {
  uint8_t* tiles = nullptr;
  WSeg seg[2];
  int N = 0, K = 0;
  int stages = 0;  // (group, k-tile) stages of the GEMV
  int chunks = 1;  // stream-K chunks (fixed per matrix)
  int64_t bytes = 0;
};

struct Layer {
  Mat qkv, o, gu, down;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* bqkv = nullptr;
};

// Per-forward dynamic parameters, copied host -> device once per forward.
struct StepDev {
  int tokens[kMaxRows];
  int positions[kMaxRows];
  int slots[kMaxRows];
  unsigned long long anc[kMaxRows];
  int step[2];  // P (keys before the new rows), P + M
  unsigned epoch;  // forward counter: value of this forward's completion flags and exchanged words
  int pad;
  // Tensor parallelism: value every rank's logits arrival counter reaches
  // once this forward's LM-head rows have all arrived (forwards with logits
  // so far x the head's 128-row groups).
  unsigned long long logits_target;
};

// Source of one weight part while building a fused matrix.
struct Part {
  const uint8_t* src = nullptr;  // raw GGUF rows
  bool on_device = false;
  int fmt = 0;
  int rows = 0;
};

// Stream-K chunk count for a GEMV of `stages` stages: one chunk per resident
// CTA of the 1-8 row instantiation (SPEC_B200_CHUNKS overrides), at most one
// per stage.
int choose_chunks(int stages, int resident_ctas);
// Partial-sum slots a matrix's split reduction needs (chunks + groups).
inline int partial_slots(const Mat& m) { return m.chunks + m.seg[0].groups + m.seg[1].groups; }

// What a launch path that brings its own scratch needs to run one standalone
// matmul of an uploaded weight (spec_qweight).  Filling it allocates nothing.
struct QmatmulLaunch {
  QmvParams p;           // weight segments, rows, splits, M, output; scratch pointers null
  int fmt_set = 0;       // forward-kernel format set of the weight
  int device = 0;
  int l2_ahead = 0;      // L2 run-ahead stages of the weight's context (SPEC_B200_L2_AHEAD)
  cudaStream_t stream = nullptr;  // the weight's own stream
};

// Makes `device` current for the lifetime of the guard and restores the
// caller's current device afterwards.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != device) cudaSetDevice(device);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};

// Reads the 16-byte device error word `err_dev` after the work on `s` (the
// stream is synchronised here), clears it on the device, and turns a
// recorded wait timeout into SPEC_ERR_TIMEOUT (an index a kernel rejected
// into SPEC_ERR_INVALID) with the record written into msg[cap].  Allocates
// nothing.
int take_device_error(unsigned* err_dev, cudaStream_t s, char* msg, size_t cap);

}  // namespace specb200

struct spec_qweight;

namespace specb200 {

// Fills `out` for y[M][N] = x[M][K] . W^T into y_dev.  Returns false for a
// null weight.
bool qweight_launch_desc(spec_qweight* w, int M, float* y_dev, QmatmulLaunch* out);
// Sets the message spec_last_error(NULL) returns on this thread (error paths).
void set_thread_error(const char* msg);

}  // namespace specb200
