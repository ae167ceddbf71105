// Verify-step attention: split-KV flash decode over the rollback KV cache with
// causal or tree (ancestor-mask) visibility, GQA rows grouped per KV head.
//
// Replaces, for the verify step, the reference's
//   Tensor::cat KV append + repeat_kv + q.k^T * scale + bias + softmax + .v
// (crates/speculate/src/model/quantized_llama_local.rs:107-136, causal bias
//  :332-350; crates/speculate/src/model/llama_local.rs:235-269) and the tree
// bias of crates/speculate/src/tree.rs:220-264 (key j of the n new rows is
// visible to row i iff j is an ancestor-or-self of i; all prefix keys are
// visible).
//
// Layout: q [n_kv][R][hd] with row r = m*G + g (token m, query head kv*G+g);
// K/V cache [n_kv][t_max][hd]; the n new keys live at slots [P, P+n).
// Split s covers absolute keys [s*C, (s+1)*C): splits are aligned to absolute
// positions, so a row's arithmetic does not depend on how many rows share the
// call (M-invariance).  Keys >= P+n are zero-filled and masked.
#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kKeyBlock = 16;

template <int HD>
struct AttnSmem {
  static constexpr int STRIDE = HD + 8;  // halves; padding breaks bank conflicts
};

template <int HD, bool BF16>
__global__ void __launch_bounds__(128) attn_split_kernel(const __grid_constant__ AttnParams p) {
  constexpr int STR = AttnSmem<HD>::STRIDE;
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem_raw[];
  pdl_launch_dependents();
  const int C = p.chunk;
  uint16_t* Ks = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* Vs = Ks + (size_t)C * STR;
  uint16_t* Qs = Vs + (size_t)C * STR;  // [warps][16][STR]

  const int split = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = p.step[0], Ttot = p.step[1];
  const int k0 = split * C;
  if (k0 >= Ttot) return;

  const uint16_t* kbase = reinterpret_cast<const uint16_t*>(p.kcache) + (size_t)kvh * p.t_max * HD;
  const uint16_t* vbase = reinterpret_cast<const uint16_t*>(p.vcache) + (size_t)kvh * p.t_max * HD;
  // Prefix keys (< P) were written by earlier forwards: fetch them before
  // waiting on the QKV kernel that appends the new keys.
  for (int i = tid; i < C * CH; i += blockDim.x) {
    const int kr = i / CH, c = i % CH, key = k0 + kr;
    if (key < P) {
      cp_async16(Ks + kr * STR + c * 8, kbase + (size_t)key * HD + c * 8, true);
      cp_async16(Vs + kr * STR + c * 8, vbase + (size_t)key * HD + c * 8, true);
    }
  }
  cp_async_commit();
  pdl_wait();
  for (int i = tid; i < C * CH; i += blockDim.x) {
    const int kr = i / CH, c = i % CH, key = k0 + kr;
    if (key >= P) {
      const bool ok = key < Ttot;
      cp_async16(Ks + kr * STR + c * 8, ok ? kbase + (size_t)key * HD + c * 8 : kbase, ok);
      cp_async16(Vs + kr * STR + c * 8, ok ? vbase + (size_t)key * HD + c * 8 : vbase, ok);
    }
  }
  cp_async_commit();

  const int M = p.M, G = p.G, R = M * G;
  const int RT = (R + 15) / 16;
  const uint16_t* qg = reinterpret_cast<const uint16_t*>(p.q) + (size_t)kvh * R * HD;
  uint16_t* qw = Qs + (size_t)warp * 16 * STR;
  const int g = lane >> 2, t = lane & 3;
  const int nsplit_max = p.max_splits;

  cp_async_wait<0>();
  __syncthreads();

  for (int rt = warp; rt < RT; rt += kAttnWarps) {
    // Stage this warp's 16 query rows.
    for (int i = lane; i < 16 * CH; i += 32) {
      const int rr = i / CH, c = i % CH, r = rt * 16 + rr;
      const bool ok = r < R;
      cp_async16(qw + rr * STR + c * 8, ok ? qg + (size_t)r * HD + c * 8 : qg, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();

    // Per-lane rows: g and g+8 of this tile.
    int rowv[2];
    unsigned long long anc[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rt * 16 + g + 8 * h;
      rowv[h] = r;
      anc[h] = (r < R) ? p.anc[r / G] : 0ull;
    }
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int kb = 0; kb < C; kb += kKeyBlock) {
      // S = Q K^T for 16 rows x 16 keys.
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t a[4], b[4];
        {
          const int q = lane >> 3, rr = (q & 1) * 8 + (lane & 7), col = kk * 16 + (q >> 1) * 8;
          ldsm_x4(a, qw + rr * STR + col);
        }
        {
          const int q = lane >> 3, key = kb + (q >> 1) * 8 + (lane & 7), col = kk * 16 + (q & 1) * 8;
          ldsm_x4(b, Ks + key * STR + col);
        }
        if constexpr (BF16) {
          mma_bf16(s[0], a[0], a[1], a[2], a[3], b[0], b[1], s[0][0], s[0][1], s[0][2], s[0][3]);
          mma_bf16(s[1], a[0], a[1], a[2], a[3], b[2], b[3], s[1][0], s[1][1], s[1][2], s[1][3]);
        } else {
          mma_f16(s[0], a[0], a[1], a[2], a[3], b[0], b[1], s[0][0], s[0][1], s[0][2], s[0][3]);
          mma_f16(s[1], a[0], a[1], a[2], a[3], b[2], b[3], s[1][0], s[1][1], s[1][2], s[1][3]);
        }
      }
      // Mask, scale (log2 domain), block max.
      float bmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int h = i >> 1;
          const int key = k0 + kb + nt * 8 + 2 * t + (i & 1);
          bool vis = key < P;
          if (!vis) {
            const int j = key - P;
            vis = (key < Ttot) && (j < 64) && ((anc[h] >> j) & 1ull);
          }
          const float v = vis ? s[nt][i] * p.scale_log2 : -INFINITY;
          s[nt][i] = v;
          bmax[h] = fmaxf(bmax[h], v);
        }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        bmax[h] = fmaxf(bmax[h], __shfl_xor_sync(0xffffffffu, bmax[h], 1));
        bmax[h] = fmaxf(bmax[h], __shfl_xor_sync(0xffffffffu, bmax[h], 2));
      }
      float alpha[2], muse[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float mnew = fmaxf(mrow[h], bmax[h]);
        muse[h] = (mnew == -INFINITY) ? 0.f : mnew;
        alpha[h] = exp2f(mrow[h] - muse[h]);
        mrow[h] = mnew;
      }
      float psum[2] = {0.f, 0.f};
      uint32_t pa[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pv[i] = exp2f(s[nt][i] - muse[i >> 1]);
        }
        if constexpr (BF16) {
          const __nv_bfloat162 lo = __floats2bfloat162_rn(pv[0], pv[1]);
          const __nv_bfloat162 hi = __floats2bfloat162_rn(pv[2], pv[3]);
          pa[nt * 2 + 0] = *reinterpret_cast<const uint32_t*>(&lo);
          pa[nt * 2 + 1] = *reinterpret_cast<const uint32_t*>(&hi);
          psum[0] += __low2float(lo) + __high2float(lo);
          psum[1] += __low2float(hi) + __high2float(hi);
        } else {
          const __half2 lo = __floats2half2_rn(pv[0], pv[1]);
          const __half2 hi = __floats2half2_rn(pv[2], pv[3]);
          pa[nt * 2 + 0] = *reinterpret_cast<const uint32_t*>(&lo);
          pa[nt * 2 + 1] = *reinterpret_cast<const uint32_t*>(&hi);
          psum[0] += __low2float(lo) + __high2float(lo);
          psum[1] += __low2float(hi) + __high2float(hi);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 1);
        psum[h] += __shfl_xor_sync(0xffffffffu, psum[h], 2);
        lrow[h] = lrow[h] * alpha[h] + psum[h];
      }
      // A operand of P.V: rows g/g+8 x keys 2t..(+8) in mma A order.
      const uint32_t a0 = pa[0], a1 = pa[1], a2 = pa[2], a3 = pa[3];
#pragma unroll
      for (int j = 0; j < HD / 8; j += 2) {
        uint32_t b[4];
        const int q = lane >> 3, key = kb + (q & 1) * 8 + (lane & 7), col = j * 8 + (q >> 1) * 8;
        ldsm_x4_trans(b, Vs + key * STR + col);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          float* oo = o[j + jj];
          oo[0] *= alpha[0];
          oo[1] *= alpha[0];
          oo[2] *= alpha[1];
          oo[3] *= alpha[1];
          float d[4] = {oo[0], oo[1], oo[2], oo[3]};
          if constexpr (BF16)
            mma_bf16(d, a0, a1, a2, a3, b[jj * 2], b[jj * 2 + 1], d[0], d[1], d[2], d[3]);
          else
            mma_f16(d, a0, a1, a2, a3, b[jj * 2], b[jj * 2 + 1], d[0], d[1], d[2], d[3]);
          oo[0] = d[0];
          oo[1] = d[1];
          oo[2] = d[2];
          oo[3] = d[3];
        }
      }
    }
    // Write this split's partial state.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rowv[h];
      if (r < R) {
        const size_t base = ((size_t)kvh * nsplit_max + split) * R + r;
        if (t == 0) {
          p.part_ml[base * 2 + 0] = mrow[h];
          p.part_ml[base * 2 + 1] = lrow[h];
        }
        float* po = p.part_o + base * HD;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
          *reinterpret_cast<float2*>(po + j * 8 + 2 * t) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
        }
      }
    }
    __syncwarp();
  }
}

SPEC_DEV void frag_store_a(uint32_t* frag, int nt_total, int m, int k, uint16_t bits) {
  const int s = k >> 4, kk = k & 15, nt = m >> 3, g = m & 7;
  const int t = (kk & 7) >> 1, slot = kk >> 3, lo = kk & 1;
  const size_t hidx = ((size_t)((s * nt_total + nt) * 32 + g * 4 + t)) * 4 + slot * 2 + lo;
  reinterpret_cast<uint16_t*>(frag)[hidx] = bits;
}

// One warp per (kv head, row r): merge the splits and emit the O-projection
// operand for columns (kv*G + g)*hd + [0, hd).  Split weights are formed with
// lane-strided partial sums and a fixed butterfly; the output rows are
// accumulated in split order.  Splits past a row's last visible key carry
// weight exactly 0, so the result does not depend on how many rows share the
// call.
template <int HD>
__global__ void __launch_bounds__(128) attn_combine_kernel(const __grid_constant__ AttnParams p, int nt_total) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = p.M * p.G;
  const int item = blockIdx.x * 4 + warp;
  if (item >= p.n_kv * R) return;
  const int kvh = item / R, r = item % R;
  const int m = r / p.G, gq = r % p.G;
  const int Ttot = p.step[1];
  const int ns = (Ttot + p.chunk - 1) / p.chunk;
  const size_t base0 = (size_t)kvh * p.max_splits * R + r;  // + s * R
  float mx = -INFINITY;
  for (int s = lane; s < ns; s += 32) mx = fmaxf(mx, __ldcg(p.part_ml + (base0 + (size_t)s * R) * 2));
  mx = warp_max(mx);
  float lsum = 0.f;
  for (int s = lane; s < ns; s += 32) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + (base0 + (size_t)s * R) * 2));
    const float w = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - mx);
    lsum += w * ml.y;
  }
  lsum = warp_sum(lsum);
  constexpr int C = HD / 32;
  float acc[C];
#pragma unroll
  for (int c = 0; c < C; ++c) acc[c] = 0.f;
  for (int s0 = 0; s0 < ns; s0 += 32) {
    float wl = 0.f;
    if (s0 + lane < ns) {
      const float msv = __ldcg(p.part_ml + (base0 + (size_t)(s0 + lane) * R) * 2);
      wl = (msv == -INFINITY) ? 0.f : exp2f(msv - mx);
    }
    const int cnt = ns - s0 < 32 ? ns - s0 : 32;
    for (int j0 = 0; j0 < cnt; j0 += 8) {
      float v[8][C];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (j0 + q < cnt) {
          const float* po = p.part_o + (base0 + (size_t)(s0 + j0 + q) * R) * HD;
#pragma unroll
          for (int c = 0; c < C; ++c) v[q][c] = __ldcg(po + c * 32 + lane);
        }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float w = __shfl_sync(0xffffffffu, wl, (j0 + q) & 31);
        if (j0 + q < cnt) {
#pragma unroll
          for (int c = 0; c < C; ++c) acc[c] += w * v[q][c];
        }
      }
    }
  }
  const float inv = (lsum > 0.f) ? 1.f / lsum : 0.f;
  const int head = kvh * p.G + gq;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int k = head * HD + c * 32 + lane;
    const float v = acc[c] * inv;
    float back;
    uint16_t bits;
    if (p.act_bf16) {
      const __nv_bfloat16 b = __float2bfloat16_rn(v);
      back = __bfloat162float(b);
      bits = __bfloat16_as_ushort(b);
    } else {
      const __half h = __float2half_rn(v);
      back = __half2float(h);
      bits = __half_as_ushort(h);
    }
    frag_store_a(p.frag, nt_total, m, k, bits);
    float s16 = back;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
    const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
    const int w16 = 8 * nt_total;
    if ((lane & 15) == 0) p.xsum16[(size_t)(k >> 4) * w16 + m] = kXSum16Seed * s16;
    if (lane == 0) p.xsum32[(size_t)(k >> 5) * w16 + m] = kXSum32Seed * s32;
  }
}

template <int HD, bool BF16>
cudaError_t launch_hd(const AttnParams& p, int nt, cudaStream_t s, bool pdl) {
  constexpr int STR = AttnSmem<HD>::STRIDE;
  const size_t smem = ((size_t)2 * p.chunk + kAttnWarps * 16) * STR * 2;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<HD, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, p.n_kv, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_split_kernel<HD, BF16>, p);
  if (e != cudaSuccess) return e;
  const int items = p.n_kv * p.M * p.G;
  cudaLaunchConfig_t cfg2 = cfg;
  cfg2.gridDim = dim3((items + 3) / 4, 1, 1);
  cfg2.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg2, attn_combine_kernel<HD>, p, nt);
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, int nt, cudaStream_t s, bool pdl) {
  if (p.M < 1 || p.M > kMaxRows || p.chunk % kKeyBlock) return cudaErrorInvalidValue;
  if (p.hd == 128) return p.act_bf16 ? launch_hd<128, true>(p, nt, s, pdl) : launch_hd<128, false>(p, nt, s, pdl);
  if (p.hd == 64) return p.act_bf16 ? launch_hd<64, true>(p, nt, s, pdl) : launch_hd<64, false>(p, nt, s, pdl);
  return cudaErrorNotSupported;
}

}  // namespace specb200
