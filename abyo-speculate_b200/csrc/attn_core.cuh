// Verify-step attention, the per-CTA pieces: one split of the flash-decode
// (a KV head's keys [split*C, split*C + C)) and the merge of a row's splits
// into the O-projection operand.  The standalone attention kernels
// (attention.cu) and the attention ops of the persistent forward kernel
// (qgemv.cu) both run these functions, so the two paths compute the same bits.
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
// call (M-invariance).  Key blocks past the last key are skipped: for every
// row they are fully masked, and a fully masked block leaves (m, l, o)
// exactly unchanged, so skipping them changes no bit.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {
namespace attn {

constexpr int kWarps = 4;                  // warps of a split unit (128 threads); tree verifies use 8
constexpr int kKeyBlock = kAttnKeyBlock;   // keys per online-softmax step (two 16-key MMA tiles)

template <int HD>
struct Smem {
  static constexpr int STRIDE = HD + 8;  // halves; padding breaks bank conflicts
};

// Shared-memory bytes of a split unit of `w` warps that stages `kp` keys per pass.
__host__ __device__ constexpr int unit_smem_bytes(int hd, int kp, int w = kWarps) {
  return (2 * kp + w * 16) * (hd + 8) * 2;
}

SPEC_DEV void sync128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Barrier 1 over the W warps of a split unit.
template <int W>
SPEC_DEV void sync_unit() {
  if constexpr (W == 4) sync128();
  else asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory");
}

// One split unit, run by threads 0 .. 32W-1 of the CTA (all of them call it
// with the same arguments).  `kp` keys (a multiple of kKeyBlock) are staged
// per pass in `smem` (unit_smem_bytes(HD, kp, W) bytes).  wait_inputs() is called
// once by all the unit's threads, after the prefix keys' loads are issued and before
// any load of what the QKV projection of this forward wrote (new keys, q
// rows).  Returns false when the split holds no key (nothing written).
// DS = warps per 16-row tile (1 or 2), each accumulating P.V for HD/DS head
// columns; S and the softmax state are formed the same way by each, so the
// result does not depend on DS.
template <int HD, bool BF16, int DS, int W = kWarps, class Wait>
SPEC_DEV bool split_unit(const AttnParams& p, int split, int kvh, uint8_t* smem, int kp, Wait&& wait_inputs) {
  static_assert(DS == 1 || DS == 2, "one or two warps per row tile");
  constexpr int STR = Smem<HD>::STRIDE;
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  const int C = p.chunk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = p.step[0], Ttot = p.step[1];
  const int k0 = split * C;
  if (k0 >= Ttot) return false;
  // Keys this split computes: up to the block holding the last key.
  const int kend = min(C, (Ttot - k0 + kKeyBlock - 1) / kKeyBlock * kKeyBlock);
  const int npass = (kend + kp - 1) / kp;

  uint16_t* Ks = reinterpret_cast<uint16_t*>(smem);
  uint16_t* Vs = Ks + (size_t)kp * STR;
  uint16_t* Qs = Vs + (size_t)kp * STR;  // [warps][16][STR]
  const uint16_t* kbase = reinterpret_cast<const uint16_t*>(p.kcache) + (size_t)kvh * p.t_max * HD;
  const uint16_t* vbase = reinterpret_cast<const uint16_t*>(p.vcache) + (size_t)kvh * p.t_max * HD;

  const int M = p.M, G = p.G, R = M * G;
  const int RT = (R + 15) / 16;
  const uint16_t* qg = reinterpret_cast<const uint16_t*>(p.q) + (size_t)kvh * R * HD;
  uint16_t* qw = Qs + (size_t)warp * 16 * STR;
  const int g = lane >> 2, t = lane & 3;
  const int nsplit_max = p.max_splits;
  bool waited = false;

  // Stages keys [a, b) of the split (smem rows 0..b-a).  Keys >= Ttot are
  // zero-filled (masked, and finite for P.V).  The first call fetches the
  // prefix keys (< P, written by earlier forwards) before waiting on the
  // projection that appends the new keys.
  auto load_kv = [&](int a, int b) {
    const int n = (b - a) * CH;
    const bool first = !waited;
    if (first) {
      for (int i = tid; i < n; i += W * 32) {
        const int kr = i / CH, c = i % CH, key = k0 + a + kr;
        if (key < P) {
          cp_async16(Ks + kr * STR + c * 8, kbase + (size_t)key * HD + c * 8, true);
          cp_async16(Vs + kr * STR + c * 8, vbase + (size_t)key * HD + c * 8, true);
        }
      }
      cp_async_commit();
      wait_inputs();
      waited = true;
    }
    for (int i = tid; i < n; i += W * 32) {
      const int kr = i / CH, c = i % CH, key = k0 + a + kr;
      if (!first || key >= P) {
        const bool ok = key < Ttot;
        cp_async16(Ks + kr * STR + c * 8, ok ? kbase + (size_t)key * HD + c * 8 : kbase, ok);
        cp_async16(Vs + kr * STR + c * 8, ok ? vbase + (size_t)key * HD + c * 8 : vbase, ok);
      }
    }
  };

  // With DS = 2, warps 2i and 2i+1 share row tile rt0 + i: both form S and
  // the softmax state (identical arithmetic), each accumulates P.V for half
  // of the head dimensions (dims [dh*HD/2, dh*HD/2 + HD/2)).
  constexpr int HALF = HD / 8 / DS;  // 8-column blocks per warp
  constexpr int TPR = W / DS;        // row tiles per round
  const int dh = DS == 2 ? (warp & 1) : 0;
  bool first_load = true;
  for (int rt0 = 0; rt0 < RT; rt0 += TPR) {
    const int rt = rt0 + warp / DS;  // this warp's 16-row tile (idle when >= RT)
    unsigned long long anc[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rt * 16 + g + 8 * h;
      anc[h] = (rt < RT && r < R) ? p.anc[r / G] : 0ull;
    }
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    float o[HALF][4];
#pragma unroll
    for (int j = 0; j < HALF; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int ps = 0; ps < npass; ++ps) {
      const int a = ps * kp, b = min(kend, a + kp);
      if (first_load) {
        load_kv(a, b);
        first_load = false;
      } else if (npass > 1) {
        sync_unit<W>();  // every warp is done with the previous pass's keys
        load_kv(a, b);
      }
      if (ps == 0 && rt < RT) {
        // Stage this warp's 16 query rows.
        for (int i = lane; i < 16 * CH; i += 32) {
          const int rr = i / CH, c = i % CH, r = rt * 16 + rr;
          const bool ok = r < R;
          cp_async16(qw + rr * STR + c * 8, ok ? qg + (size_t)r * HD + c * 8 : qg, ok);
        }
      }
      cp_async_commit();
      cp_async_wait<0>();
      sync_unit<W>();
      if (rt >= RT) continue;

      for (int kb = a; kb < b; kb += kKeyBlock) {
        const int sr = kb - a;  // smem row of the block
        // S = Q K^T for 16 rows x 32 keys: two 16-key halves x two 8-key
        // n-tiles, four independent MMA chains over the head dimension.
        float s[2][2][4];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) s[h2][nt][0] = s[h2][nt][1] = s[h2][nt][2] = s[h2][nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          uint32_t a4[4];
          {
            const int q = lane >> 3, rr = (q & 1) * 8 + (lane & 7), col = kk * 16 + (q >> 1) * 8;
            ldsm_x4(a4, qw + rr * STR + col);
          }
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t b4[4];
            const int q = lane >> 3, key = sr + h2 * 16 + (q >> 1) * 8 + (lane & 7), col = kk * 16 + (q & 1) * 8;
            ldsm_x4(b4, Ks + key * STR + col);
            float(&s0)[4] = s[h2][0];
            float(&s1)[4] = s[h2][1];
            if constexpr (BF16) {
              mma_bf16(s0, a4[0], a4[1], a4[2], a4[3], b4[0], b4[1], s0[0], s0[1], s0[2], s0[3]);
              mma_bf16(s1, a4[0], a4[1], a4[2], a4[3], b4[2], b4[3], s1[0], s1[1], s1[2], s1[3]);
            } else {
              mma_f16(s0, a4[0], a4[1], a4[2], a4[3], b4[0], b4[1], s0[0], s0[1], s0[2], s0[3]);
              mma_f16(s1, a4[0], a4[1], a4[2], a4[3], b4[2], b4[3], s1[0], s1[1], s1[2], s1[3]);
            }
          }
        }
        // Mask, scale (log2 domain), block max.
        float bmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int h = i >> 1;
              const int key = k0 + kb + h2 * 16 + nt * 8 + 2 * t + (i & 1);
              bool vis = key < P;
              if (!vis) {
                const int j = key - P;
                vis = (key < Ttot) && (j < 64) && ((anc[h] >> j) & 1ull);
              }
              const float v = vis ? s[h2][nt][i] * p.scale_log2 : -INFINITY;
              s[h2][nt][i] = v;
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
        uint32_t pa[2][4];  // A operand of P.V per 16-key half: rows g/g+8 x keys 2t..(+8)
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            float pv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = exp2f(s[h2][nt][i] - muse[i >> 1]);
            if constexpr (BF16) {
              const __nv_bfloat162 lo = __floats2bfloat162_rn(pv[0], pv[1]);
              const __nv_bfloat162 hi = __floats2bfloat162_rn(pv[2], pv[3]);
              pa[h2][nt * 2 + 0] = *reinterpret_cast<const uint32_t*>(&lo);
              pa[h2][nt * 2 + 1] = *reinterpret_cast<const uint32_t*>(&hi);
              psum[0] += __low2float(lo) + __high2float(lo);
              psum[1] += __low2float(hi) + __high2float(hi);
            } else {
              const __half2 lo = __floats2half2_rn(pv[0], pv[1]);
              const __half2 hi = __floats2half2_rn(pv[2], pv[3]);
              pa[h2][nt * 2 + 0] = *reinterpret_cast<const uint32_t*>(&lo);
              pa[h2][nt * 2 + 1] = *reinterpret_cast<const uint32_t*>(&hi);
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
#pragma unroll
        for (int j = 0; j < HALF; ++j) {
          o[j][0] *= alpha[0];
          o[j][1] *= alpha[0];
          o[j][2] *= alpha[1];
          o[j][3] *= alpha[1];
        }
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
          for (int j = 0; j < HALF; j += 2) {
            uint32_t b4[4];
            const int q = lane >> 3, key = sr + h2 * 16 + (q & 1) * 8 + (lane & 7);
            const int col = (dh * HALF + j) * 8 + (q >> 1) * 8;
            ldsm_x4_trans(b4, Vs + key * STR + col);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              float(&d)[4] = o[j + jj];
              if constexpr (BF16)
                mma_bf16(d, pa[h2][0], pa[h2][1], pa[h2][2], pa[h2][3], b4[jj * 2], b4[jj * 2 + 1], d[0], d[1], d[2],
                         d[3]);
              else
                mma_f16(d, pa[h2][0], pa[h2][1], pa[h2][2], pa[h2][3], b4[jj * 2], b4[jj * 2 + 1], d[0], d[1], d[2],
                        d[3]);
            }
          }
        }
      }
    }
    if (rt < RT) {
      // This split's partial state for the warp's rows and columns.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = rt * 16 + g + 8 * h;
        if (r < R) {
          const size_t base = ((size_t)kvh * nsplit_max + split) * R + r;
          if (t == 0 && dh == 0) {
            p.part_ml[base * 2 + 0] = mrow[h];
            p.part_ml[base * 2 + 1] = lrow[h];
          }
          float* po = p.part_o + base * HD + dh * (HD / DS);
#pragma unroll
          for (int j = 0; j < HALF; ++j)
            *reinterpret_cast<float2*>(po + j * 8 + 2 * t) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
        }
      }
    }
    if (rt0 + TPR < RT) sync_unit<W>();  // the next round restages the q rows
  }
  return true;
}

SPEC_DEV void frag_store_a(uint32_t* frag, int nt_total, int m, int k, uint16_t bits, int bf16) {
  reinterpret_cast<uint16_t*>(frag)[operand_half_index(nt_total, m, k, bf16 != 0)] = bits;
}

// One warp per item = (KV head, row r, columns [32q, 32q + 32) of the head):
// merge the splits and emit those columns of the O-projection operand.  Split
// weights are formed with lane-strided partial sums and a fixed butterfly; a
// column is accumulated in split order, with up to 16 splits' loads in flight.
// Splits past a row's last visible key carry weight exactly 0, so the result
// does not depend on how many rows share the call.  Split partials are read
// through L2 (they were written by other CTAs).
template <int HD>
SPEC_DEV void combine_item(const AttnParams& p, int nt_total, int item, int lane) {
  constexpr int Q = HD / 32;
  const int R = p.M * p.G;
  if (item >= attn_combine_items(p.n_kv, R, HD)) return;
  const int cq = item % Q, rk = item / Q;
  const int kvh = rk / R, r = rk % R;
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
  float acc = 0.f;
  const int col = cq * 32 + lane;
  for (int s0 = 0; s0 < ns; s0 += 32) {
    float wl = 0.f;
    if (s0 + lane < ns) {
      const float msv = __ldcg(p.part_ml + (base0 + (size_t)(s0 + lane) * R) * 2);
      wl = (msv == -INFINITY) ? 0.f : exp2f(msv - mx);
    }
    const int cnt = ns - s0 < 32 ? ns - s0 : 32;
    constexpr int B = 16;  // splits in flight per batch
    for (int j0 = 0; j0 < cnt; j0 += B) {
      float v[B];
#pragma unroll
      for (int q = 0; q < B; ++q)
        v[q] = (j0 + q < cnt) ? __ldcg(p.part_o + (base0 + (size_t)(s0 + j0 + q) * R) * HD + col) : 0.f;
#pragma unroll
      for (int q = 0; q < B; ++q) {
        const float w = __shfl_sync(0xffffffffu, wl, (j0 + q) & 31);
        if (j0 + q < cnt) acc += w * v[q];
      }
    }
  }
  const float inv = (lsum > 0.f) ? 1.f / lsum : 0.f;
  const int head = kvh * p.G + gq;
  const int k = p.col_off + head * HD + col;
  const float v = acc * inv;
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
  frag_store_a(p.frag, nt_total, m, k, bits, p.act_bf16);
  float s16 = back;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
  const int w16 = 8 * nt_total;
  if ((lane & 15) == 0) p.xsum16[(size_t)(k >> 4) * w16 + m] = kXSum16Seed * s16;
  if (lane == 0) p.xsum32[(size_t)(k >> 5) * w16 + m] = kXSum32Seed * s32;
}

}  // namespace attn
}  // namespace specb200
