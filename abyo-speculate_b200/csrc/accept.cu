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

// block_seq_sum over values computed while they are staged: f(i) for
// i in [0, n).  Same chunking and add order as block_seq_sum.
template <class F>
SPEC_DEV void stage_chunk_of(F f, int base, int len, float* buf, bool skip_warp0) {
  const int t0 = skip_warp0 ? 32 : 0;
  if ((int)threadIdx.x < t0) return;
  for (int i = threadIdx.x - t0; i < len; i += blockDim.x - t0) buf[i] = f(base + i);
}

template <class F>
SPEC_DEV float block_seq_sum_of(F f, int n, float* buf, float* bcast) {
  float s = 0.f;
  const int nc = (n + kSeqChunk - 1) / kSeqChunk;
  if (nc > 0) stage_chunk_of(f, 0, min(kSeqChunk, n), buf, false);
  __syncthreads();
  for (int c = 0; c < nc; ++c) {
    const int base = c * kSeqChunk, len = min(kSeqChunk, n - base);
    float* cur = buf + (c & 1) * kSeqChunk;
    if (c + 1 < nc)
      stage_chunk_of(f, base + kSeqChunk, min(kSeqChunk, n - base - kSeqChunk), buf + ((c + 1) & 1) * kSeqChunk,
                     true);
    if (threadIdx.x == 0) s = add_chunk(s, cur, len);
    __syncthreads();
  }
  if (threadIdx.x == 0) *bcast = s;
  __syncthreads();
  s = *bcast;
  __syncthreads();
  return s;
}

// Thread 0: s += buf[0..len) in order, every partial sum stored to
// out[0..len) (16-byte aligned).  Same add sequence as add_chunk.
SPEC_DEV float add_chunk_pref(float s, const float* buf, int len, float* out) {
  const int n16 = len & ~15;
  if (n16) {
    float4 a0 = *reinterpret_cast<const float4*>(buf), a1 = *reinterpret_cast<const float4*>(buf + 4),
           a2 = *reinterpret_cast<const float4*>(buf + 8), a3 = *reinterpret_cast<const float4*>(buf + 12);
    for (int i = 0; i < n16; i += 16) {
      const float4 b[4] = {a0, a1, a2, a3};
      if (i + 16 < n16) {
        a0 = *reinterpret_cast<const float4*>(buf + i + 16);
        a1 = *reinterpret_cast<const float4*>(buf + i + 20);
        a2 = *reinterpret_cast<const float4*>(buf + i + 24);
        a3 = *reinterpret_cast<const float4*>(buf + i + 28);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 o;
        s = __fadd_rn(s, b[q].x); o.x = s;
        s = __fadd_rn(s, b[q].y); o.y = s;
        s = __fadd_rn(s, b[q].z); o.z = s;
        s = __fadd_rn(s, b[q].w); o.w = s;
        *reinterpret_cast<float4*>(out + i + 4 * q) = o;
      }
    }
  }
  for (int i = n16; i < len; ++i) {
    s = __fadd_rn(s, buf[i]);
    out[i] = s;
  }
  return s;
}

// tokens.rs:99-120 over probs[0..n) with the uniform u01 (block-wide; every
// thread receives the index); -1 on an invalid distribution.  The reference
// sums the row, then scans it again accumulating from 0 in the same order:
// the scan's running sums are exactly the sum's partial sums.  So one
// sequential pass (thread 0, chunks staged by the other warps as in
// block_seq_sum) stores every partial sum to pref[0..n), the staging threads
// note the first invalid element (non-finite or negative; the reference
// checks each before adding it), and the first index whose partial sum
// exceeds u = u01 * sum is then found by all threads at once.  pref may be
// probs itself (a chunk is overwritten only after it has been staged).
SPEC_DEV int block_sample(const float* probs, int n, float u01, float* pref, float* buf, float* bcast,
                          int* ibcast, int* ibad) {
  if (threadIdx.x == 0) {
    *ibcast = INT_MAX;
    *ibad = INT_MAX;
  }
  __syncthreads();
  auto stage = [&](int base, int len, float* dst, bool skip_warp0) {
    const int t0 = skip_warp0 ? 32 : 0;
    if ((int)threadIdx.x < t0) return;
    for (int i = threadIdx.x - t0; i < len; i += blockDim.x - t0) {
      const float v = probs[base + i];
      if (!isfinite(v) || v < 0.f) atomicMin(ibad, base + i);
      dst[i] = v;
    }
  };
  float s = 0.f;
  const int nc = (n + kSeqChunk - 1) / kSeqChunk;
  if (nc > 0) stage(0, min(kSeqChunk, n), buf, false);
  __syncthreads();
  for (int c = 0; c < nc; ++c) {
    const int base = c * kSeqChunk, len = min(kSeqChunk, n - base);
    float* cur = buf + (c & 1) * kSeqChunk;
    if (c + 1 < nc) stage(base + kSeqChunk, min(kSeqChunk, n - base - kSeqChunk), buf + ((c + 1) & 1) * kSeqChunk, true);
    if (threadIdx.x == 0) s = add_chunk_pref(s, cur, len, pref + base);
    __syncthreads();
  }
  if (threadIdx.x == 0) *bcast = s;
  __syncthreads();
  const float sum = *bcast;
  const int bad = *ibad;
  if (!(sum > 0.f) || !isfinite(sum)) {
    __syncthreads();
    return -1;
  }
  const float u = __fmul_rn(u01, sum);
  // First index with u < partial sum; a thread stops at its first hit, and
  // no index at or beyond the block's current best is worth reading.
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (u < pref[i]) {
      atomicMin(ibcast, i);
      break;
    }
  }
  __syncthreads();
  const int hit = *ibcast;
  __syncthreads();
  if (bad != INT_MAX && (hit == INT_MAX || bad <= hit)) return -1;
  return hit != INT_MAX ? hit : n - 1;
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
  // The exponentials are computed (and kept in the row) by the warps that
  // stage each chunk for thread 0's sequential sum.
  const float s = block_seq_sum_of(
      [&](int i) {
        const float e = exp_f32_cr(__fmul_rn(__fsub_rn(row[i], mx), inv_t));
        row[i] = e;
        return e;
      },
      V, s_buf, &s_sum);
  if (threadIdx.x == 0 && (!(s > 0.f) || !isfinite(s))) atomicCAS(status, 0, REJ_ERR_SOFTMAX);
  for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = __fdiv_rn(row[i], s);
}

// The round's walk (single CTA).  p: [k+1][V] target probabilities,
// q: [k][V] draft probabilities, r: [V] scratch.
__global__ void __launch_bounds__(kRejThreads) rejection_walk_kernel(const float* p, const float* q, float* r,
                                                                     const RejStep* st, int V, int* out) {
  __shared__ int s_i, s_n, s_used, s_status, s_reject, s_idx, s_bad;
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
        const int idx = block_sample(r, V, st->uniforms[s_used], r, s_buf, &s_sum, &s_idx, &s_bad);
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
      const int idx = block_sample(p + (size_t)k * V, V, st->uniforms[s_used], r, s_buf, &s_sum, &s_idx, &s_bad);
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

// ---- typical acceptance (methods/medusa.rs:424-445) -----------------------
// f32::ln modelled as the correctly rounded log of the f32 argument (log in
// double, one rounding), as exp is above.
SPEC_DEV float ln_f32_cr(float x) { return (float)log((double)x); }

// One CTA per tree row that has children.  softmax: NaN-skipping max, then
// e_i = exp(l_i - max) and their sequential f32 sum; p_i = e_i / sum.
// entropy: sequential f32 sum of (-p) * ln(p) over p > 0 (skipped elements
// contribute -0.0, which leaves every partial sum unchanged).  threshold =
// max(epsilon, delta * exp(-entropy)); a child passes iff p(token) >=
// threshold.  A row whose mass is non-positive or non-finite rejects every
// child (the reference returns false).  Nothing is stored but the flags.
__global__ void __launch_bounds__(kRejThreads) typical_accept_kernel(const float* rows, int V, TypicalTree t,
                                                                     int* accept) {
  const int r = blockIdx.x;
  bool has_child = false;
  for (int i = 1; i < t.n; ++i) has_child |= t.par[i] == r;
  if (!has_child) return;  // uniform across the block
  const float* row = rows + (size_t)r * V;
  __shared__ float red[kRejThreads / 32];
  __shared__ float s_sum;
  __shared__ __align__(16) float s_buf[2 * kSeqChunk];
  const float mx = block_max(row, V, red);
  const float s = block_seq_sum_of([&](int i) { return exp_f32_cr(__fsub_rn(row[i], mx)); }, V, s_buf, &s_sum);
  const bool valid = s > 0.f && isfinite(s);
  float thr = 0.f;
  if (valid) {
    const float h = block_seq_sum_of(
        [&](int i) {
          const float p = __fdiv_rn(exp_f32_cr(__fsub_rn(row[i], mx)), s);
          return p > 0.f ? __fmul_rn(-p, ln_f32_cr(p)) : -0.f;
        },
        V, s_buf, &s_sum);
    thr = fmaxf(t.epsilon, __fmul_rn(t.delta, exp_f32_cr(-h)));
  }
  for (int i = threadIdx.x; i < t.n; i += blockDim.x) {
    if (i < 1 || t.par[i] != r) continue;
    int ok = 0;
    if (valid) ok = __fdiv_rn(exp_f32_cr(__fsub_rn(row[t.tok[i]], mx)), s) >= thr;
    accept[i] = ok;
  }
}

}  // namespace

cudaError_t launch_typical_accept(const float* rows, int V, const TypicalTree& t, int* accept, cudaStream_t s) {
  if (t.n < 1 || t.n > kMaxRows || V < 1) return cudaErrorInvalidValue;
  typical_accept_kernel<<<t.n, kRejThreads, 0, s>>>(rows, V, t, accept);
  return cudaGetLastError();
}

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
