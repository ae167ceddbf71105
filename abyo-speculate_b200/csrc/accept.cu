// Rejection-sampling acceptance of one vanilla speculative round on the
// device, over the k+1 target logits rows the verify forward left in HBM.
//
// Restates, with the reference's float32 operations in the reference's order:
//   crates/speculate/src/sampling/tokens.rs:14-55  softmax_with_temperature
//     (t == 0: one-hot first-max argmax; else e = exp((l - max) * (1/t)),
//      sum = sequential f32 sum, p = e / sum; error if sum <= 0 or not finite)
//   tokens.rs:99-120  sample_from_distribution (sum = sequential f32 sum,
//      u = gen::<f32>() * sum, linear f32 cumulative scan, first i with
//      u < acc, fallback to the last index)
//   crates/speculate/src/methods/vanilla.rs:59-73  modified_rejection_step
//      (accept iff q <= 0 or u <= min(p / q, 1))
//   vanilla.rs:83-106  adjusted_distribution (max(p - q, 0) / sequential sum;
//      error if the mass is <= 0)
//   vanilla.rs:172-210  the round: one uniform per verified position, then one
//      resample on reject, or one bonus sample from row k when all k drafts
//      were accepted and the token budget allows.
//
// Every sum and scan that the reference runs sequentially runs on one thread
// here, so the f32 rounding sequence is the reference's; max, exp and the
// divisions are element-wise and run in parallel.  exp is evaluated in double
// and rounded once to f32 (the correctly rounded value of exp on the f32
// argument).
#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {

namespace {

constexpr int kRejThreads = 1024;

SPEC_DEV float exp_f32_cr(float x) { return (float)exp((double)x); }

// The row is staged through shared memory in chunks, double-buffered: warps
// 1.. load chunk c+1 while thread 0 alone adds (or scans) chunk c in index
// order, so the f32 rounding sequence is the sequential one.
constexpr int kSeqChunk = 4096;  // floats per staged chunk (16 KB; two buffers)

SPEC_DEV void stage_chunk(const float* x, int base, int len, float* buf, bool skip_warp0) {
  const int t0 = skip_warp0 ? 32 : 0;
  if ((int)threadIdx.x < t0) return;
  for (int i = threadIdx.x - t0; i < len; i += blockDim.x - t0) buf[i] = x[base + i];
}

// Thread 0: s += buf[0..len) in order.  The next 16 elements are loaded
// while the current 16 are added.
SPEC_DEV float add_chunk(float s, const float* buf, int len) {
  const int n16 = len & ~15;
  if (n16) {
    float4 a0 = *reinterpret_cast<const float4*>(buf), a1 = *reinterpret_cast<const float4*>(buf + 4),
           a2 = *reinterpret_cast<const float4*>(buf + 8), a3 = *reinterpret_cast<const float4*>(buf + 12);
    for (int i = 0; i < n16; i += 16) {
      float4 b0 = a0, b1 = a1, b2 = a2, b3 = a3;
      if (i + 16 < n16) {
        a0 = *reinterpret_cast<const float4*>(buf + i + 16);
        a1 = *reinterpret_cast<const float4*>(buf + i + 20);
        a2 = *reinterpret_cast<const float4*>(buf + i + 24);
        a3 = *reinterpret_cast<const float4*>(buf + i + 28);
      }
      s = __fadd_rn(s, b0.x); s = __fadd_rn(s, b0.y); s = __fadd_rn(s, b0.z); s = __fadd_rn(s, b0.w);
      s = __fadd_rn(s, b1.x); s = __fadd_rn(s, b1.y); s = __fadd_rn(s, b1.z); s = __fadd_rn(s, b1.w);
      s = __fadd_rn(s, b2.x); s = __fadd_rn(s, b2.y); s = __fadd_rn(s, b2.z); s = __fadd_rn(s, b2.w);
      s = __fadd_rn(s, b3.x); s = __fadd_rn(s, b3.y); s = __fadd_rn(s, b3.z); s = __fadd_rn(s, b3.w);
    }
  }
  for (int i = n16; i < len; ++i) s = __fadd_rn(s, buf[i]);
  return s;
}

// Sequential float32 sum of x[0..n) (Rust `iter().sum::<f32>()`); every
// thread of the block calls it and receives the sum.  buf: 2 * kSeqChunk.
SPEC_DEV float block_seq_sum(const float* x, int n, float* buf, float* bcast) {
  float s = 0.f;
  const int nc = (n + kSeqChunk - 1) / kSeqChunk;
  if (nc > 0) stage_chunk(x, 0, min(kSeqChunk, n), buf, false);
  __syncthreads();
  for (int c = 0; c < nc; ++c) {
    const int base = c * kSeqChunk, len = min(kSeqChunk, n - base);
    float* cur = buf + (c & 1) * kSeqChunk;
    if (c + 1 < nc)
      stage_chunk(x, base + kSeqChunk, min(kSeqChunk, n - base - kSeqChunk), buf + ((c + 1) & 1) * kSeqChunk, true);
    if (threadIdx.x == 0) s = add_chunk(s, cur, len);
    __syncthreads();
  }
  if (threadIdx.x == 0) *bcast = s;
  __syncthreads();
  s = *bcast;
  __syncthreads();
  return s;
}

// tokens.rs:99-120 over probs[0..n) with the uniform u01 (block-wide; every
// thread receives the index); -1 on an invalid distribution.
SPEC_DEV int block_sample(const float* probs, int n, float u01, float* buf, float* bcast, int* ibcast) {
  const float sum = block_seq_sum(probs, n, buf, bcast);
  if (!(sum > 0.f) || !isfinite(sum)) return -1;
  const float u = __fmul_rn(u01, sum);
  float acc = 0.f;
  const int nc = (n + kSeqChunk - 1) / kSeqChunk;
  stage_chunk(probs, 0, min(kSeqChunk, n), buf, false);
  if (threadIdx.x == 0) *ibcast = -2;  // -2: not found yet
  __syncthreads();
  for (int c = 0; c < nc; ++c) {
    const int base = c * kSeqChunk, len = min(kSeqChunk, n - base);
    const float* cur = buf + (c & 1) * kSeqChunk;
    if (c + 1 < nc)
      stage_chunk(probs, base + kSeqChunk, min(kSeqChunk, n - base - kSeqChunk), buf + ((c + 1) & 1) * kSeqChunk,
                  true);
    if (threadIdx.x == 0) {
      // 16 elements per step, the next 16 loaded ahead.  The running sum
      // advances unconditionally; the answer is the first
      // index whose running sum exceeds u, unless an invalid element comes at
      // or before it (the reference checks each element before adding it).
      // Neither record feeds back into the add chain.
      int hit = -1, bad = -1;
      auto step = [&](float p, int idx) {
        const bool invalid = !isfinite(p) || p < 0.f;
        bad = (bad < 0 && invalid) ? idx : bad;
        acc = __fadd_rn(acc, p);
        hit = (hit < 0 && u < acc) ? idx : hit;
      };
      const int n16 = len & ~15;
      int i = 0;
      if (n16) {
        float4 a0 = *reinterpret_cast<const float4*>(cur), a1 = *reinterpret_cast<const float4*>(cur + 4),
               a2 = *reinterpret_cast<const float4*>(cur + 8), a3 = *reinterpret_cast<const float4*>(cur + 12);
        for (; i < n16 && (bad | hit) < 0; i += 16) {
          const float4 b0 = a0, b1 = a1, b2 = a2, b3 = a3;
          if (i + 16 < n16) {
            a0 = *reinterpret_cast<const float4*>(cur + i + 16);
            a1 = *reinterpret_cast<const float4*>(cur + i + 20);
            a2 = *reinterpret_cast<const float4*>(cur + i + 24);
            a3 = *reinterpret_cast<const float4*>(cur + i + 28);
          }
          step(b0.x, i + 0); step(b0.y, i + 1); step(b0.z, i + 2); step(b0.w, i + 3);
          step(b1.x, i + 4); step(b1.y, i + 5); step(b1.z, i + 6); step(b1.w, i + 7);
          step(b2.x, i + 8); step(b2.y, i + 9); step(b2.z, i + 10); step(b2.w, i + 11);
          step(b3.x, i + 12); step(b3.y, i + 13); step(b3.z, i + 14); step(b3.w, i + 15);
        }
      }
      for (; i < len && (bad | hit) < 0; ++i) step(cur[i], i);
      if (bad >= 0 && (hit < 0 || bad <= hit)) *ibcast = -1;
      else if (hit >= 0) *ibcast = base + hit;
    }
    __syncthreads();
    const int found = *ibcast;
    if (found != -2) return found;  // uniform: read after the barrier by every thread
    __syncthreads();
  }
  return n - 1;
}

// Block-wide first-max argmax (tokens.rs:26-36 fold) of row[0..V).
SPEC_DEV int block_argmax(const float* row, int V, unsigned long long* red) {
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v == v) {
      unsigned u = __float_as_uint(v);
      u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
      const unsigned long long key = ((unsigned long long)u << 32) | (unsigned)(~i);
      best = max(best, key);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = max(best, red[w]);
    red[0] = best;
  }
  __syncthreads();
  best = red[0];
  __syncthreads();
  return best ? (int)(~(unsigned)(best & 0xffffffffull)) : 0;
}

// Block-wide max with f32::max semantics (NaN operands are ignored).
SPEC_DEV float block_max(const float* row, int V, float* red) {
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, row[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    red[0] = m;
  }
  __syncthreads();
  m = red[0];
  __syncthreads();
  return m;
}

// One CTA per target row: logits -> probabilities in place.
__global__ void __launch_bounds__(kRejThreads) target_softmax_kernel(float* rows, int V, float temperature,
                                                                     int* status) {
  float* row = rows + (size_t)blockIdx.x * V;
  __shared__ unsigned long long red64[kRejThreads / 32];
  __shared__ float red[kRejThreads / 32];
  __shared__ float s_sum;
  __shared__ __align__(16) float s_buf[2 * kSeqChunk];
  if (temperature == 0.f) {
    const int am = block_argmax(row, V, red64);
    for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = i == am ? 1.f : 0.f;
    return;
  }
  const float inv_t = __fdiv_rn(1.f, temperature);
  const float mx = block_max(row, V, red);
  for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = exp_f32_cr(__fmul_rn(__fsub_rn(row[i], mx), inv_t));
  __syncthreads();
  const float s = block_seq_sum(row, V, s_buf, &s_sum);
  if (threadIdx.x == 0 && (!(s > 0.f) || !isfinite(s))) atomicCAS(status, 0, REJ_ERR_SOFTMAX);
  for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = __fdiv_rn(row[i], s);
}

// The round's walk (single CTA).  p: [k+1][V] target probabilities,
// q: [k][V] draft probabilities, r: [V] scratch.
__global__ void __launch_bounds__(kRejThreads) rejection_walk_kernel(const float* p, const float* q, float* r,
                                                                     const RejStep* st, int V, int* out) {
  __shared__ int s_i, s_n, s_used, s_status, s_reject, s_idx;
  __shared__ float s_sum;
  __shared__ __align__(16) float s_buf[2 * kSeqChunk];
  const int k = st->k;
  if (threadIdx.x == 0) {
    s_n = 0;
    s_used = 0;
    s_status = out[2];
    s_reject = -1;
    s_i = 0;
  }
  __syncthreads();
  if (s_status != 0) {
    if (threadIdx.x == 0) out[0] = out[1] = 0;
    return;
  }
  // Accept tests (scalar); stop at the first rejection.
  if (threadIdx.x == 0) {
    int n = 0, used = 0;
    for (int i = 0; i < k; ++i) {
      const int tok = st->drafts[i];
      if (used >= st->n_uniforms) {
        s_status = REJ_ERR_UNIFORMS;
        break;
      }
      const float u = st->uniforms[used++];
      const float qx = q[(size_t)i * V + tok], px = p[(size_t)i * V + tok];
      const bool accept = qx <= 0.f || u <= fminf(__fdiv_rn(px, qx), 1.f);
      if (accept) {
        out[4 + n++] = tok;
        if (n >= st->budget) break;
      } else {
        s_reject = i;
        break;
      }
    }
    s_n = n;
    s_used = used;
  }
  __syncthreads();
  if (s_status == 0 && s_reject >= 0) {
    // vanilla.rs:83-106 then tokens.rs:99-120 on the adjusted distribution.
    const int i = s_reject;
    const float* pi = p + (size_t)i * V;
    const float* qi = q + (size_t)i * V;
    for (int j = threadIdx.x; j < V; j += blockDim.x) r[j] = fmaxf(__fsub_rn(pi[j], qi[j]), 0.f);
    __syncthreads();
    const float s = block_seq_sum(r, V, s_buf, &s_sum);
    if (!(s > 0.f) || !isfinite(s)) {
      if (threadIdx.x == 0) s_status = REJ_ERR_ADJUSTED;
    } else {
      for (int j = threadIdx.x; j < V; j += blockDim.x) r[j] = __fdiv_rn(r[j], s);
      __syncthreads();
      if (s_used >= st->n_uniforms) {
        if (threadIdx.x == 0) s_status = REJ_ERR_UNIFORMS;
      } else {
        const int idx = block_sample(r, V, st->uniforms[s_used], s_buf, &s_sum, &s_idx);
        if (threadIdx.x == 0) {
          ++s_used;
          if (idx < 0) s_status = REJ_ERR_DISTRIBUTION;
          else out[4 + s_n++] = idx;
        }
      }
    }
  } else if (s_status == 0 && s_n == k && s_n < st->budget) {
    // All k accepted: bonus token from row k.
    if (s_used >= st->n_uniforms) {
      if (threadIdx.x == 0) s_status = REJ_ERR_UNIFORMS;
    } else {
      const int idx = block_sample(p + (size_t)k * V, V, st->uniforms[s_used], s_buf, &s_sum, &s_idx);
      if (threadIdx.x == 0) {
        ++s_used;
        if (idx < 0) s_status = REJ_ERR_DISTRIBUTION;
        else out[4 + s_n++] = idx;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    out[0] = s_n;
    out[1] = s_used;
    out[2] = s_status;
  }
}

}  // namespace

cudaError_t launch_rejection(float* rows, const float* q, float* r, const RejStep* st, int k, int V,
                             float temperature, int* out, cudaStream_t s) {
  if (k < 0 || k + 1 > kMaxRows || V < 1) return cudaErrorInvalidValue;
  target_softmax_kernel<<<k + 1, kRejThreads, 0, s>>>(rows, V, temperature, out + 2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  rejection_walk_kernel<<<1, kRejThreads, 0, s>>>(rows, q, r, st, V, out);
  return cudaGetLastError();
}

}  // namespace specb200
