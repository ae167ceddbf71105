// Small kernels around the verify step: embedding gather-dequant, KV-cache
// reorder (accepted-path commit), final-norm hidden rows, row argmax, and the
// seeded on-device generator for synthetic quantized weights.
#include "common.cuh"
#include "kernels.cuh"

#include <math.h>

namespace specb200 {

namespace {

SPEC_DEV float h2f16(uint16_t b) { return __half2float(__ushort_as_half(b)); }
SPEC_DEV uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

SPEC_DEV void k4_sm(const uint8_t* q, int j, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Element k of a GGUF row, with the same f32 operation order as the GGUF
// reference decode (no fused multiply-add), so the embedding rows are
// bit-identical to a host dequantization.
SPEC_DEV float deq_elem(const uint8_t* row, int fmt, int k) {
  switch (fmt) {
    case WF_Q4_K:
    case WF_Q5_K: {
      const int bb = fmt == WF_Q4_K ? 144 : 176;
      const uint8_t* b = row + (size_t)(k >> 8) * bb;
      const int kk = k & 255, c = kk >> 6, l = kk & 31, hi = (kk & 63) >> 5;
      int sc, m;
      k4_sm(b + 4, 2 * c + hi, sc, m);
      const float d = h2f16(rd_u16(b)), dmin = h2f16(rd_u16(b + 2));
      const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
      int q;
      if (fmt == WF_Q4_K) {
        const uint8_t byte = b[16 + 32 * c + l];
        q = hi ? (byte >> 4) : (byte & 15);
      } else {
        const uint8_t byte = b[48 + 32 * c + l];
        q = (hi ? (byte >> 4) : (byte & 15)) + (((b[16 + l] >> (2 * c + hi)) & 1) ? 16 : 0);
      }
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case WF_Q6_K: {
      const uint8_t* b = row + (size_t)(k >> 8) * 210;
      const int kk = k & 255, n = kk >> 7, r = kk & 127, j = r >> 5, l = r & 31;
      const uint8_t lb = b[64 * n + l + (j & 1) * 32];
      const int lo = (j < 2) ? (lb & 15) : (lb >> 4);
      const int hi = (b[128 + 32 * n + l] >> (2 * j)) & 3;
      const int q = (lo | (hi << 4)) - 32;
      const int is = l / 16;
      const float d = h2f16(rd_u16(b + 208));
      const float sc = (float)(int8_t)b[192 + 8 * n + is + 2 * j];
      return __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
    case WF_Q8_0: {
      const uint8_t* b = row + (size_t)(k >> 5) * 34;
      return __fmul_rn(h2f16(rd_u16(b)), (float)(int8_t)b[2 + (k & 31)]);
    }
    case WF_F32:
      return reinterpret_cast<const float*>(row)[k];
    case WF_F16:
      return h2f16(reinterpret_cast<const uint16_t*>(row)[k]);
    case WF_BF16: {
      const uint32_t bits = (uint32_t)reinterpret_cast<const uint16_t*>(row)[k] << 16;
      return __uint_as_float(bits);
    }
  }
  return 0.f;
}

SPEC_DEV void frag_store_m(uint32_t* frag, int nt_total, int m, int k, uint16_t bits, int bf16) {
  reinterpret_cast<uint16_t*>(frag)[operand_half_index(nt_total, m, k, bf16 != 0)] = bits;
}

// grid (H/128, M), 128 threads: one column each.
__global__ void __launch_bounds__(128) embed_kernel(const __grid_constant__ EmbedParams p, int nt_total) {
  __shared__ float s_red[4];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = blockIdx.x, m = blockIdx.y;
  const int n = grp * 128 + tid;
  const int tok = p.tokens[m];
  float v = 0.f;
  if (tok >= 0 && tok < p.V) {
    const size_t row_bytes = (size_t)(p.H / fmt_block_elems(p.fmt)) * fmt_block_bytes(p.fmt);
    v = deq_elem(p.table + (size_t)tok * row_bytes, p.fmt, n);
  } else if (tid == 0) {
    atomicOr(p.err, DEV_ERR_BAD_ARGUMENT);
  }
  p.h[(size_t)m * p.H + n] = v;
  const float sq = warp_sum(v * v);
  if (lane == 0) s_red[warp] = sq;
  // operand of the first GEMV: f16/bf16(h * attn_norm)
  const float x = p.norm ? v * p.norm[n] : v;
  float back;
  uint16_t bits;
  if (p.act_bf16) {
    const __nv_bfloat16 b = __float2bfloat16_rn(x);
    back = __bfloat162float(b);
    bits = __bfloat16_as_ushort(b);
  } else {
    const __half h = __float2half_rn(x);
    back = __half2float(h);
    bits = __half_as_ushort(h);
  }
  frag_store_m(p.frag, nt_total, m, n, bits, p.act_bf16);
  float s16 = back;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
  const int w16 = 8 * nt_total;
  if ((lane & 15) == 0) p.xsum16[(size_t)(n >> 4) * w16 + m] = kXSum16Seed * s16;
  if (lane == 0) p.xsum32[(size_t)(n >> 5) * w16 + m] = kXSum32Seed * s32;
  __syncthreads();
  if (tid == 0) p.ss_out[grp * kSsStride + m] = s_red[0] + s_red[1] + s_red[2] + s_red[3];
}

// Reorder: for every (layer, arena K/V, kv head) copy rows src[i] -> tmp, then
// tmp -> dst[i].  One CTA per (layer*2 + arena, kv head).
__global__ void kv_gather_kernel(uint16_t* kcache, uint16_t* vcache, int n_kv, int t_max, int hd,
                                 const int* src, const int* dst, int n, uint16_t* tmp) {
  const int la = blockIdx.x, h = blockIdx.y;
  const int layer = la >> 1, arena = la & 1;
  uint16_t* base = (arena ? vcache : kcache) + ((size_t)layer * n_kv + h) * t_max * hd;
  uint16_t* tb = tmp + ((size_t)la * n_kv + h) * (size_t)n * hd;
  for (int i = threadIdx.x; i < n * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    tb[i] = base[(size_t)src[r] * hd + d];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    base[(size_t)dst[r] * hd + d] = tb[i];
  }
}

__global__ void final_hidden_kernel(const float* h, const float* ss, int groups, float inv_dim, float eps,
                                    const float* norm, int H, float* out) {
  const int m = blockIdx.x;
  float ms = 0.f;
  for (int q = 0; q < groups; ++q) ms += ss[q * kSsStride + m];
  const float r = 1.f / sqrtf(ms * inv_dim + eps);
  for (int n = threadIdx.x; n < H; n += blockDim.x) out[(size_t)m * H + n] = h[(size_t)m * H + n] * r * norm[n];
}

// First-max argmax (strict '>' scan order), one CTA per row.
// Row argmax with the first-max tie break (a sequential scan with strict >):
// every (row, chunk) CTA folds its slice into one 64-bit key (order-preserving
// float bits, then the complemented index, so a larger key is a larger value
// or, on a tie, a smaller index) and merges it with atomicMax; the CTA that
// arrives last for a row decodes the key and clears the slot and counter for
// the next call.  The max of a set of keys does not depend on arrival order.
// NaN entries are skipped; a row of only NaN yields index 0.  -0.0 keys as
// +0.0 (the reference's `>` treats them as equal, so the lower index wins).
SPEC_DEV unsigned long long argmax_key(float v, int i) {
  unsigned u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)(~i);
}
SPEC_DEV float argmax_key_value(unsigned long long k) {
  unsigned u = (unsigned)(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}

__global__ void __launch_bounds__(256) row_argmax_kernel(const float* logits, int V, int per_cta,
                                                         unsigned long long* slots, int* counters, int* out_idx,
                                                         float* out_val) {
  const int row = blockIdx.y;
  const float* x = logits + (size_t)row * V;
  const int start = blockIdx.x * per_cta, end = min(V, start + per_cta);
  unsigned long long best = 0ull;
  for (int i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float v = __ldg(x + i);
    if (v == v) best = max(best, argmax_key(v, i));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ unsigned long long sb[8];
  __shared__ bool s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sb[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = max(best, sb[w]);
    atomicMax(slots + row, best);
    __threadfence();
    s_last = atomicAdd(counters + row, 1) == (int)gridDim.x - 1;
    if (s_last) {
      __threadfence();
      const unsigned long long k = atomicExch(slots + row, 0ull);
      counters[row] = 0;
      out_idx[row] = k ? (int)(~(unsigned)(k & 0xffffffffull)) : 0;
      if (out_val) out_val[row] = k ? argmax_key_value(k) : -INFINITY;
    }
  }
}

// ---- top-k over a logits row (methods/medusa.rs:477-487) ------------------
// Values descending, ties by ascending index: exactly the order of the
// argmax keys above, so the top k of a row are its k largest keys (NaN
// entries key as 0, below every value).  Stage 1: each CTA stages a chunk's
// keys in shared memory and extracts its k largest in k rounds of "largest
// key below the previous one"; stage 2 does the same over the chunks'
// candidates.  Keys are unique (the index is part of them), so each round
// is one block-wide max.
constexpr int kTopKChunk = 4096;

SPEC_DEV unsigned long long block_max_u64(unsigned long long v, unsigned long long* sb) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sb[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) v = max(v, sb[w]);
    sb[0] = v;
  }
  __syncthreads();
  v = sb[0];
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(256) topk_chunk_kernel(const float* logits, int V, int k, unsigned long long* part) {
  __shared__ unsigned long long keys[kTopKChunk];
  __shared__ unsigned long long sb[8];
  const int row = blockIdx.y, chunk = blockIdx.x;
  const int start = chunk * kTopKChunk, n = min(kTopKChunk, V - start);
  const float* x = logits + (size_t)row * V + start;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __ldg(x + i);
    keys[i] = v == v ? argmax_key(v, start + i) : 0ull;
  }
  __syncthreads();
  unsigned long long* out = part + ((size_t)row * gridDim.x + chunk) * k;
  unsigned long long prev = ~0ull;
  for (int r = 0; r < k; ++r) {
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long kk = keys[i];
      if (kk < prev && kk > best) best = kk;
    }
    best = block_max_u64(best, sb);
    if (threadIdx.x == 0) out[r] = best;
    prev = best;
  }
}

__global__ void __launch_bounds__(256) topk_merge_kernel(const unsigned long long* part, int chunks, int k,
                                                         int* ids, float* vals) {
  __shared__ unsigned long long sb[8];
  const int row = blockIdx.x, n = chunks * k;
  const unsigned long long* c = part + (size_t)row * n;
  unsigned long long prev = ~0ull;
  for (int r = 0; r < k; ++r) {
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long kk = c[i];
      if (kk < prev && kk > best) best = kk;
    }
    best = block_max_u64(best, sb);
    if (threadIdx.x == 0) {
      ids[row * k + r] = best ? (int)(~(unsigned)(best & 0xffffffffull)) : -1;
      vals[row * k + r] = best ? argmax_key_value(best) : __int_as_float(0x7fc00000);
    }
    prev = best;
  }
}

// ---- EAGLE draft block glue (methods/eagle.rs:390-427) ----------------------
// x2 = concat(hidden, embed(token)) with the token read from device memory
// (the previous draft step's top-1), so a draft-depth loop runs without host
// round trips.  grid (2H / 128), 128 threads.
__global__ void __launch_bounds__(128) eagle_concat_kernel(const uint8_t* table, int fmt, int H, int V,
                                                           const int* tok, const float* hidden, float* x2,
                                                           unsigned* err) {
  const int n = blockIdx.x * 128 + threadIdx.x;
  if (n >= 2 * H) return;
  if (n < H) {
    x2[n] = hidden[n];
    return;
  }
  const int t = *tok;
  float v = 0.f;
  if (t >= 0 && t < V) {
    const size_t row_bytes = (size_t)(H / fmt_block_elems(fmt)) * fmt_block_bytes(fmt);
    v = deq_elem(table + (size_t)t * row_bytes, fmt, n - H);
  } else if (n == H) {
    atomicOr(err, DEV_ERR_BAD_ARGUMENT);
  }
  x2[n] = v;
}

// h2 = t + h; xn = RMSNorm(h2) * w (post_attention_layernorm).  One CTA.
__global__ void __launch_bounds__(256) eagle_resid_norm_kernel(const float* t, const float* h, const float* w, int H,
                                                               float eps, float* h2, float* xn) {
  __shared__ float red[8];
  __shared__ float s_r;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = t[i] + h[i];
    h2[i] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a += red[i];
    s_r = 1.f / sqrtf(a / (float)H + eps);
  }
  __syncthreads();
  const float r = s_r;
  for (int i = threadIdx.x; i < H; i += blockDim.x) xn[i] = h2[i] * r * w[i];
}

__global__ void eagle_add_kernel(const float* a, const float* b, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] + b[i];
}

// A Medusa residual block's update (methods/medusa.rs:571-575):
// out = x + SiLU(y), y = the block's linear output (bias included).
__global__ void medusa_res_kernel(const float* x, const float* y, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = y[i];
    out[i] = x[i] + v / (1.f + expf(-v));
  }
}

// log(sum(exp(x - max))) + max over one row (NaN entries skipped).  One CTA.
__global__ void __launch_bounds__(1024) row_lse_kernel(const float* x, int V, float* out) {
  __shared__ float red[32];
  __shared__ float s_m;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, x[i]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a = fmaxf(a, red[i]);
    s_m = a;
  }
  __syncthreads();
  const float mx = s_m;
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = x[i];
    if (v == v) s += expf(v - mx);
  }
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) a += red[i];
    *out = logf(a) + mx;
  }
}

// ---- seeded synthetic weights --------------------------------------------
SPEC_DEV uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
SPEC_DEV float gauss(uint64_t seed, uint64_t idx) {
  const uint64_t r = splitmix64(seed ^ splitmix64(idx));
  const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = ((float)((r >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
  return sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
}

SPEC_DEV uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// One GGUF block assembled in registers (up to 212 bytes as 53 words), then
// written out with 16-bit stores: every block base is 2-byte aligned
// (cudaMalloc alignment, even block sizes) and no byte of global memory is
// read back or written twice.  (Building the block with byte read-modify-
// writes in global memory left the low byte of Q6_K's d and of Q4_K's dmin
// wrong on B200, which scaled Q6_K weights by about 0.79 and biased Q4_K
// weights by +0.003.)
struct BlockBytes {
  uint32_t w[53];
  SPEC_DEV void clear() {
#pragma unroll
    for (int i = 0; i < 53; ++i) w[i] = 0u;
  }
  SPEC_DEV void set(int i, uint32_t v) { w[i >> 2] |= (v & 0xffu) << (8 * (i & 3)); }
  SPEC_DEV void store(uint8_t* out, int bytes) const {
    uint16_t* o = reinterpret_cast<uint16_t*>(out);
    for (int i = 0; i < bytes / 2; ++i) o[i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
  }
};

// One thread per block of the row-major [rows][K] matrix.
__global__ void synth_quant_kernel(uint8_t* raw, int fmt, int rows, int K, uint64_t seed, float sigma,
                                   int row_offset) {
  const int be = fmt_block_elems(fmt), bb = fmt_block_bytes(fmt);
  const int nbr = K / be;
  const size_t blk = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (blk >= (size_t)rows * nbr) return;
  const int r = (int)(blk / nbr), c = (int)(blk % nbr);
  uint8_t* out = raw + blk * bb;
  const uint64_t base = ((uint64_t)(r + row_offset) * (uint64_t)K) + (uint64_t)c * be;
  if (fmt == WF_BF16 || fmt == WF_F16 || fmt == WF_F32) {
    const float x = sigma * gauss(seed, base);
    if (fmt == WF_BF16) {
      *reinterpret_cast<uint16_t*>(out) = __bfloat16_as_ushort(__float2bfloat16_rn(x));
    } else if (fmt == WF_F16) {
      *reinterpret_cast<uint16_t*>(out) = f2h_bits(x);
    } else {
      *reinterpret_cast<float*>(out) = x;
    }
    return;
  }
  BlockBytes B;
  B.clear();
  if (fmt == WF_Q8_0) {
    float x[32], amax = 0.f;
    for (int i = 0; i < 32; ++i) {
      x[i] = sigma * gauss(seed, base + i);
      amax = fmaxf(amax, fabsf(x[i]));
    }
    const uint16_t db = f2h_bits(amax / 127.f);
    const float d = h2f16(db);
    B.set(0, db & 0xff);
    B.set(1, db >> 8);
    for (int i = 0; i < 32; ++i) {
      const float q = d > 0.f ? rintf(x[i] / d) : 0.f;
      B.set(2 + i, (uint8_t)(int8_t)fminf(fmaxf(q, -127.f), 127.f));
    }
    B.store(out, bb);
    return;
  }
  float x[256];
  for (int i = 0; i < 256; ++i) x[i] = sigma * gauss(seed, base + i);
  if (fmt == WF_Q6_K) {
    float scale[16], dmax = 0.f;
    for (int s = 0; s < 16; ++s) {
      float am = 0.f;
      for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(x[16 * s + i]));
      scale[s] = am / 31.f;
      dmax = fmaxf(dmax, scale[s]);
    }
    const uint16_t db = f2h_bits(dmax / 127.f);
    const float d = h2f16(db);
    B.set(208, db & 0xff);
    B.set(209, db >> 8);
    for (int s = 0; s < 16; ++s) {
      const int sc = d > 0.f ? (int)fminf(fmaxf(rintf(scale[s] / d), 0.f), 127.f) : 0;
      B.set(192 + s, (uint8_t)(int8_t)sc);
      const float se = d * (float)sc;
      for (int i = 0; i < 16; ++i) {
        const int k = 16 * s + i;
        int q = se > 0.f ? (int)fminf(fmaxf(rintf(x[k] / se), -32.f), 31.f) : 0;
        q += 32;
        // GGUF Q6_K: half n = k / 128; within it quarter j = (k % 128) / 32 and
        // lane l: low nibble in ql[64 n + l + 32 (j & 1)] (high nibble for
        // j >= 2), top 2 bits in qh[32 n + l] at bit 2 j.
        const int n = k >> 7, rr = k & 127, j = rr >> 5, l = rr & 31;
        B.set(64 * n + l + (j & 1) * 32, (j < 2) ? (q & 15) : ((q & 15) << 4));
        B.set(128 + 32 * n + l, ((q >> 4) & 3) << (2 * j));
      }
    }
    B.store(out, bb);
    return;
  }
  // Q4_K / Q5_K
  const int levels = fmt == WF_Q4_K ? 15 : 31;
  float scale[8], mins[8], smax = 0.f, mmax = 0.f;
  for (int s = 0; s < 8; ++s) {
    float lo = 0.f, hi = -INFINITY;
    for (int i = 0; i < 32; ++i) {
      lo = fminf(lo, x[32 * s + i]);
      hi = fmaxf(hi, x[32 * s + i]);
    }
    scale[s] = (hi - lo) / levels;
    mins[s] = -lo;
    smax = fmaxf(smax, scale[s]);
    mmax = fmaxf(mmax, mins[s]);
  }
  const uint16_t db = f2h_bits(smax / 63.f), dmb = f2h_bits(mmax / 63.f);
  const float d = h2f16(db), dm = h2f16(dmb);
  B.set(0, db & 0xff);
  B.set(1, db >> 8);
  B.set(2, dmb & 0xff);
  B.set(3, dmb >> 8);
  int sc[8], mq[8];
  for (int s = 0; s < 8; ++s) {
    sc[s] = d > 0.f ? (int)fminf(fmaxf(rintf(scale[s] / d), 0.f), 63.f) : 0;
    mq[s] = dm > 0.f ? (int)fminf(fmaxf(rintf(mins[s] / dm), 0.f), 63.f) : 0;
  }
  // 6-bit (scale, min) packing of the GGUF K-quants: sub-blocks 0-3 in the low
  // 6 bits of bytes 4-7 / 8-11; sub-blocks 4-7 as low nibbles in bytes 12-15
  // and their top 2 bits in the high bits of bytes 4-11.
  for (int j = 0; j < 4; ++j) {
    B.set(4 + j, (sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    B.set(8 + j, (mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
    B.set(12 + j, (sc[j + 4] & 15) | ((mq[j + 4] & 15) << 4));
  }
  const int qoff = fmt == WF_Q4_K ? 16 : 48;
  for (int k = 0; k < 256; ++k) {
    const int s = k >> 5;
    const float se = d * (float)sc[s], ce = dm * (float)mq[s];
    const int q = se > 0.f ? (int)fminf(fmaxf(rintf((x[k] + ce) / se), 0.f), (float)levels) : 0;
    const int cc = k >> 6, l = k & 31, hi = (k & 63) >> 5;
    B.set(qoff + 32 * cc + l, (q & 15) << (hi ? 4 : 0));
    if (fmt == WF_Q5_K && (q >> 4)) B.set(16 + l, 1u << (2 * cc + hi));
  }
  B.store(out, bb);
}

// grid (ceil(K/128), M): f32 row-major activations -> operand fragments.
__global__ void __launch_bounds__(128) make_operand_kernel(const float* x, int K, int nt_total, uint32_t* frag,
                                                           float* xs16, float* xs32, int bf16) {
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.y;
  const int k = blockIdx.x * 128 + threadIdx.x;
  if (blockIdx.x * 128 + (threadIdx.x & ~31) >= K) return;  // whole warp out of range
  const float v = x[(size_t)m * K + k];
  float back;
  uint16_t bits;
  if (bf16) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    back = __bfloat162float(b);
    bits = __bfloat16_as_ushort(b);
  } else {
    const __half h = __float2half_rn(v);
    back = __half2float(h);
    bits = __half_as_ushort(h);
  }
  frag_store_m(frag, nt_total, m, k, bits, bf16);
  float s16 = back;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
  const int w16 = 8 * nt_total;
  if ((lane & 15) == 0) xs16[(size_t)(k >> 4) * w16 + m] = kXSum16Seed * s16;
  if (lane == 0) xs32[(size_t)(k >> 5) * w16 + m] = kXSum32Seed * s32;
}

__global__ void synth_vec_kernel(float* out, int n, uint64_t seed, float base, float sigma) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = base + sigma * gauss(seed, (uint64_t)i);
}

}  // namespace

cudaError_t launch_embed(const EmbedParams& p, int nt, cudaStream_t s, bool pdl) {
  if (p.H % 128 || p.M < 1 || p.M > kMaxRows) return cudaErrorInvalidValue;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.H / 128, p.M, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, embed_kernel, p, nt);
}

cudaError_t launch_kv_gather(void* kcache, void* vcache, int layers, int n_kv, int t_max, int hd, const int* src,
                             const int* dst, int n, void* tmp, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  kv_gather_kernel<<<dim3(layers * 2, n_kv), 256, 0, s>>>(reinterpret_cast<uint16_t*>(kcache),
                                                           reinterpret_cast<uint16_t*>(vcache), n_kv, t_max, hd, src,
                                                           dst, n, reinterpret_cast<uint16_t*>(tmp));
  return cudaGetLastError();
}

cudaError_t launch_make_operand(const float* x, int M, int K, int nt, uint32_t* frag, float* xsum16, float* xsum32,
                                int bf16, cudaStream_t s) {
  if (K % 32 || M < 1 || M > kMaxRows) return cudaErrorInvalidValue;
  make_operand_kernel<<<dim3((K + 127) / 128, M), 128, 0, s>>>(x, K, nt, frag, xsum16, xsum32, bf16);
  return cudaGetLastError();
}

cudaError_t launch_final_hidden(const float* h, const float* ss, int groups, float inv_dim, float eps,
                                const float* norm, int M, int H, float* out, cudaStream_t s) {
  final_hidden_kernel<<<M, 256, 0, s>>>(h, ss, groups, inv_dim, eps, norm, H, out);
  return cudaGetLastError();
}

cudaError_t launch_row_argmax(const float* logits, int rows, int V, int* out_idx, float* out_val,
                              unsigned long long* slots, int* counters, cudaStream_t s) {
  if (rows < 1 || rows > kMaxRows || V < 1) return cudaErrorInvalidValue;
  const int per_cta = 2048;
  row_argmax_kernel<<<dim3((V + per_cta - 1) / per_cta, rows), 256, 0, s>>>(logits, V, per_cta, slots, counters,
                                                                           out_idx, out_val);
  return cudaGetLastError();
}

cudaError_t launch_row_topk(const float* logits, int rows, int V, int k, unsigned long long* part, int* ids,
                            float* vals, cudaStream_t s) {
  if (rows < 1 || rows > kMaxRows || V < 1 || k < 1 || k > kMaxTopK || k > V) return cudaErrorInvalidValue;
  const int chunks = (V + kTopKChunk - 1) / kTopKChunk;
  if (chunks > kTopKMaxChunks) return cudaErrorInvalidValue;
  topk_chunk_kernel<<<dim3(chunks, rows), 256, 0, s>>>(logits, V, k, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  topk_merge_kernel<<<rows, 256, 0, s>>>(part, chunks, k, ids, vals);
  return cudaGetLastError();
}

cudaError_t launch_eagle_concat(const uint8_t* table, int fmt, int H, int V, const int* tok, const float* hidden,
                                float* x2, unsigned* err, cudaStream_t s) {
  eagle_concat_kernel<<<(2 * H + 127) / 128, 128, 0, s>>>(table, fmt, H, V, tok, hidden, x2, err);
  return cudaGetLastError();
}
cudaError_t launch_eagle_resid_norm(const float* t, const float* h, const float* w, int H, float eps, float* h2,
                                    float* xn, cudaStream_t s) {
  eagle_resid_norm_kernel<<<1, 256, 0, s>>>(t, h, w, H, eps, h2, xn);
  return cudaGetLastError();
}
cudaError_t launch_eagle_add(const float* a, const float* b, float* out, int n, cudaStream_t s) {
  eagle_add_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, b, out, n);
  return cudaGetLastError();
}
cudaError_t launch_medusa_res(const float* x, const float* y, float* out, int n, cudaStream_t s) {
  medusa_res_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, y, out, n);
  return cudaGetLastError();
}
cudaError_t launch_row_lse(const float* x, int V, float* out, cudaStream_t s) {
  row_lse_kernel<<<1, 1024, 0, s>>>(x, V, out);
  return cudaGetLastError();
}

cudaError_t launch_synth_quant(uint8_t* raw, int fmt, int rows, int K, uint64_t seed, float sigma, int row_offset,
                               cudaStream_t s) {
  const int be = fmt_block_elems(fmt);
  if (be == 0 || K % be) return cudaErrorInvalidValue;
  const size_t blocks = (size_t)rows * (K / be);
  const int th = 128;
  synth_quant_kernel<<<(unsigned)((blocks + th - 1) / th), th, 0, s>>>(raw, fmt, rows, K, seed, sigma, row_offset);
  return cudaGetLastError();
}

cudaError_t launch_synth_vec(float* out, int n, uint64_t seed, float base, float sigma, cudaStream_t s) {
  synth_vec_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, n, seed, base, sigma);
  return cudaGetLastError();
}

}  // namespace specb200
