// Dequant-MMA GEMV/small-M GEMM for GGUF Q4_K / Q5_K / Q6_K / Q8_0 and BF16
// weights: y[m][n] = sum_k W[n][k] * x[m][k] for M <= 64 activation rows.
//
// Replaces candle's `QMatMul::forward` on the verify step
// (crates/speculate/src/model/quantized_llama_local.rs:47-49,73-90,135,316-318;
//  crates/speculate/src/model/quantized_qwen2_local.rs:41-44,71-82,138,314-316)
// and the `Linear` layers of the BF16 model (llama_local.rs:235-269).
//
// Design (sm_100a):
//  * Weights are repacked at load into 16-row tiles whose bytes are already in
//    m16n8k16 A-fragment order: lane (g,t) finds, in one 32-bit word per
//    k-step, the 8 codes of rows g / g+8 at columns 2t, 2t+1, 2t+8, 2t+9.
//    Two 16-row tiles form a "pair tile" (32 rows x KT columns); one warp owns
//    a 32-row slice.  Tiles are laid out [group][k-tile][warp], so one stage
//    (128 rows x one k-tile) is a single TMA bulk copy (cp.async.bulk ->
//    shared, mbarrier completion, L2 evict-first) into a 2-3 stage ring.
//  * Codes become f16 with one LOP3 each (magic 0x6400: value = 1024 + q;
//    Q4_K / Q5_K rows g+8 take the high nibble in place, 1024 + 16q, with the
//    1/16 folded into their sub-block scales),
//    feed mma.sync with the activation fragments, and the accumulator is
//    seeded with -offset * (sum of the activations of that sub-block), so the
//    tensor core returns exactly sum(q * x) for the sub-block.  The sub-block
//    scale (and K-quant min term) is applied in f32 afterwards:
//        acc += s_row * D - c_row * xsum.
//    Products q*x are exact in the tensor core (q <= 63, x f16), so the only
//    roundings are the f16 activations and f32 accumulation.
//  * Work is split stream-K style: an op's (group, k-tile) stages are cut into
//    a fixed number of contiguous chunks, one per resident CTA.  A group cut
//    across chunks leaves one partial per piece; the CTA delivering the last
//    piece adds them in chunk order, then runs the fused epilogue.  The cut
//    depends only on the matrix, so row r's result is bit-identical for any
//    M (batched == sequential).
//  * Ops of one launch chain through per-group completion flags: a stage's
//    activations are fetched once the groups of the previous op that produce
//    its K range are done, so an op starts while the previous one finishes.
//  * Programmatic dependent launch: a CTA issues its first weight copies, then
//    waits for the previous kernel (griddepcontrol.wait) before touching
//    activations, so weight streaming overlaps the predecessor's tail.
#include "common.cuh"
#include "kernels.cuh"
#include "attn_core.cuh"

#include <stdlib.h>

#include <type_traits>

namespace specb200 {

namespace {

// ---------------------------------------------------------------------------
// Static tile geometry per format / n-tile count.
// ---------------------------------------------------------------------------
template <int F, int NT>
struct Geo {
  static constexpr int KT = fmt_kt(F);
  static constexpr int KS = KT / 16;                        // k-steps per tile
  static constexpr int PAIR = fmt_pair_bytes(F);            // weight bytes per pair tile
  static constexpr int XFRAG = KS * NT * 256;               // operand fragments per tile
  static constexpr int X32 = (F == WF_BF16) ? 0 : (KT / 32) * 8 * NT * 4;
  static constexpr int X16 = (F == WF_BF16) ? 0 : KS * 8 * NT * 4;
  static constexpr int XB = XFRAG + X32 + X16;              // operand bytes per tile
};

constexpr int kScratch = 2048;   // per-warp decoded-scale scratch (bytes)

SPEC_DEV float h2f_bits(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu))); }

// Q4_K / Q5_K: unpack sub-block b's 6-bit (scale, min) from the 12 packed
// bytes held in m.y (bytes 0-3), m.z (4-7), m.w (8-11).
SPEC_DEV void k4_scale_min(const uint4& m, int b, int& sc, int& mn) {
  if (b < 4) {
    sc = (m.y >> (8 * b)) & 63;
    mn = (m.z >> (8 * b)) & 63;
  } else {
    const int bb = b - 4;
    sc = ((m.w >> (8 * bb)) & 0xF) | (((m.y >> (8 * bb + 6)) & 3) << 4);
    mn = ((m.w >> (8 * bb + 4)) & 0xF) | (((m.z >> (8 * bb + 6)) & 3) << 4);
  }
}

SPEC_DEV uint32_t shift_signed(uint32_t v, int delta) { return delta >= 0 ? (v >> delta) : (v << (-delta)); }

// Four A registers (rows g/g+8, cols 2t..+1 / 2t+8..+9) from one word of
// eight 4-bit codes.  Rows g (a[0], a[2]) hold 1024 + code; rows g+8 (a[1],
// a[3]) are the high nibble of each byte masked in place, 1024 + 16 * code
// (exact in f16: 16 * 15 < 1024).  That saves two shifts per word; the
// sub-block scales of rows g+8 carry the 1/16 (decode_scales), which is exact.
SPEC_DEV void a_from_nibbles(uint32_t w, uint32_t (&a)[4]) {
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  a[1] = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  const uint32_t w8 = w >> 8;
  a[2] = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  a[3] = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
}

// ---------------------------------------------------------------------------
// Cooperative scale decode: lane l decodes row l of the pair tile (rows
// 0-15 = tile 0, 16-31 = tile 1) into the warp's scratch, laid out so that
// lane (g, t) later reads rows g and g+8 with one vector load.
// ---------------------------------------------------------------------------
template <int F>
SPEC_DEV void decode_scales(const uint8_t* tp, float* scr, int lane) {
  constexpr int TB = fmt_tile_bytes(F);
  const int rt = lane >> 4, ri = lane & 15;
  if constexpr (F == WF_Q4_K || F == WF_Q5_K) {
    // scr layout (floats): [0,256) s[rt][sb][g][row g | row g+8];
    // [256,384) m as f16 A-fragment words [rt][g][t][row g | row g+8];
    // [384,416) dmin[rt][row].
    constexpr int MO = (F == WF_Q4_K) ? 2048 : 2560;
    const uint4 m = *reinterpret_cast<const uint4*>(tp + rt * TB + MO + ri * 16);
    const float d = h2f_bits(m.x), dm = h2f_bits(m.x >> 16);
    int mv[8];
    // Rows 8-15 of the tile meet their codes as 16 * code (a_from_nibbles).
    const float rs = (ri >> 3) ? 0.0625f : 1.f;
#pragma unroll
    for (int sb = 0; sb < 8; ++sb) {
      int sc;
      k4_scale_min(m, sb, sc, mv[sb]);
      scr[((rt * 8 + sb) * 8 + (ri & 7)) * 2 + (ri >> 3)] = d * (float)sc * rs;
    }
    uint32_t* mw = reinterpret_cast<uint32_t*>(scr + 256);
#pragma unroll
    for (int t = 0; t < 4; ++t)
      mw[((rt * 8 + (ri & 7)) * 4 + t) * 2 + (ri >> 3)] =
          pack_half2(__int2half_rn(mv[2 * t]), __int2half_rn(mv[2 * t + 1]));
    scr[384 + rt * 16 + ri] = dm * 64.f;
  } else if constexpr (F == WF_Q6_K) {
    const uint4 sv = *reinterpret_cast<const uint4*>(tp + rt * TB + 3072 + ri * 16);
    const float d = h2f_bits(*reinterpret_cast<const uint16_t*>(tp + rt * TB + 3328 + ri * 2));
    const uint32_t w4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int b = 0; b < 16; ++b)
      scr[((rt * 16 + b) * 8 + (ri & 7)) * 2 + (ri >> 3)] = d * (float)(int8_t)((w4[b >> 2] >> (8 * (b & 3))) & 0xff);
  } else if constexpr (F == WF_Q8_0) {
    const uint2 dv = *reinterpret_cast<const uint2*>(tp + rt * TB + 2048 + ri * 8);
    const uint32_t w2[2] = {dv.x, dv.y};
#pragma unroll
    for (int b = 0; b < 4; ++b)
      scr[((rt * 4 + b) * 8 + (ri & 7)) * 2 + (ri >> 3)] = h2f_bits(w2[b >> 1] >> (16 * (b & 1)));
  }
}

// ---------------------------------------------------------------------------
// Per-format pair-tile compute.  tp: weights (shared), xs: operand stage
// (shared; fragments, then xsum32, then xsum16), scr: decoded scales.
// ---------------------------------------------------------------------------
template <int NT>
SPEC_DEV void load_bfrag(const uint8_t* xs, int kk, int lane, uint32_t (&b)[NT][2]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint2 v = *reinterpret_cast<const uint2*>(xs + (kk * NT + nt) * 256 + lane * 8);
    b[nt][0] = v.x;
    b[nt][1] = v.y;
  }
}

template <int NT>
SPEC_DEV float2 load_sum(const uint8_t* base, int blk, int nt, int lane) {
  return *reinterpret_cast<const float2*>(base + ((blk * NT + nt) * 8 + 2 * (lane & 3)) * 4);
}

// Q4_K / Q5_K.  Per sub-block b the tensor core returns D_b = sum(q * x)
// (its accumulator is seeded with -1024 * xsum_b to cancel the code offset);
// acc += s_b * D_b.  The min term sum_b m_b * xsum_b is one more exact mma per
// 16-row tile and superblock: A = the 6-bit mins (exact in f16), B = the
// sub-block sums / 64 split into f16 hi + lo parts; acc -= 64 * dmin * D_min.
template <int NT>
SPEC_DEV void tile_q45k(const uint8_t* tp, const uint8_t* xs, const float* scr, int lane, bool q5,
                        float (&acc)[2][NT][4]) {
  const int TB = q5 ? 2816 : 2304;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* x32 = xs + 16 * NT * 256;
  // B operand of the min-term mma: rows k = sub-blocks 2t, 2t+1; column g.
  uint32_t bh[NT], bl[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    // x32 holds -1024 x the sums: x (-1/65536) = the sums / 64, exactly.
    const float v0 = reinterpret_cast<const float*>(x32)[(2 * t) * 8 * NT + nt * 8 + g] * (-1.f / 65536.f);
    const float v1 = reinterpret_cast<const float*>(x32)[(2 * t + 1) * 8 * NT + nt * 8 + g] * (-1.f / 65536.f);
    const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    bh[nt] = pack_half2(h0, h1);
    bl[nt] = pack_half2(__float2half_rn(v0 - __half2float(h0)), __float2half_rn(v1 - __half2float(h1)));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // 4 k-steps = 2 sub-blocks of 32
    uint32_t bq[4][NT][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) load_bfrag<NT>(xs, 4 * j + i, lane, bq[i]);
    float2 xsum[2][NT];
#pragma unroll
    for (int sb = 0; sb < 2; ++sb)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xsum[sb][nt] = load_sum<NT>(x32, 2 * j + sb, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const uint32_t wv[4] = {qw.x, qw.y, qw.z, qw.w};
      uint32_t hw = 0;
      if (q5) hw = *reinterpret_cast<const uint32_t*>(tp + rt * TB + 2048 + j * 128 + lane * 4);
#pragma unroll
      for (int sb = 0; sb < 2; ++sb) {
        const float2 sc = *reinterpret_cast<const float2*>(scr + ((rt * 8 + 2 * j + sb) * 8 + g) * 2);
        uint32_t a[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * sb + h;
          a_from_nibbles(wv[i], a[h]);
          if (q5) {
            // The fifth bit: weight 16 (bit 4) in rows g, 256 (bit 8) in the
            // x16 rows g+8.
#pragma unroll
            for (int jj = 0; jj < 4; jj += 2) {
              a[h][jj] = lop3_or_and(a[h][jj], shift_signed(hw, 4 * i + jj - 4), 0x00100010u);
              a[h][jj + 1] = lop3_or_and(a[h][jj + 1], shift_signed(hw, 4 * i + jj + 1 - 8), 0x01000100u);
            }
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float c0 = xsum[sb][nt].x, c1 = xsum[sb][nt].y;  // already -1024 x the sums
          float d[4];
          mma_f16(d, a[0][0], a[0][1], a[0][2], a[0][3], bq[2 * sb][nt][0], bq[2 * sb][nt][1], c0, c1, c0, c1);
          mma_f16(d, a[1][0], a[1][1], a[1][2], a[1][3], bq[2 * sb + 1][nt][0], bq[2 * sb + 1][nt][1], d[0], d[1],
                  d[2], d[3]);
          float* ac = acc[rt][nt];
          ac[0] = fmaf(sc.x, d[0], ac[0]);
          ac[1] = fmaf(sc.x, d[1], ac[1]);
          ac[2] = fmaf(sc.y, d[2], ac[2]);
          ac[3] = fmaf(sc.y, d[3], ac[3]);
        }
      }
    }
  }
  const uint32_t* mw = reinterpret_cast<const uint32_t*>(scr + 256);
#pragma unroll
  for (int rt = 0; rt < 2; ++rt) {
    const uint2 am = *reinterpret_cast<const uint2*>(mw + ((rt * 8 + g) * 4 + t) * 2);
    const float dm0 = scr[384 + rt * 16 + g], dm1 = scr[384 + rt * 16 + g + 8];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float d[4];
      mma_f16(d, am.x, am.y, 0u, 0u, bh[nt], 0u, 0.f, 0.f, 0.f, 0.f);
      mma_f16(d, am.x, am.y, 0u, 0u, bl[nt], 0u, d[0], d[1], d[2], d[3]);
      float* ac = acc[rt][nt];
      ac[0] = fmaf(-dm0, d[0], ac[0]);
      ac[1] = fmaf(-dm0, d[1], ac[1]);
      ac[2] = fmaf(-dm1, d[2], ac[2]);
      ac[3] = fmaf(-dm1, d[3], ac[3]);
    }
  }
}

template <int NT>
SPEC_DEV void tile_q6k(const uint8_t* tp, const uint8_t* xs, const float* scr, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 3360;
  const int g = lane >> 2;
  const uint8_t* x16 = xs + 16 * NT * 256 + 8 * 8 * NT * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t bq[4][NT][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) load_bfrag<NT>(xs, 4 * j + i, lane, bq[i]);
    float2 xsum[4][NT];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xsum[i][nt] = load_sum<NT>(x16, 4 * j + i, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const uint32_t hw0 = *reinterpret_cast<const uint32_t*>(tp + rt * TB + 2048 + (2 * j) * 128 + lane * 4);
      const uint32_t hw1 = *reinterpret_cast<const uint32_t*>(tp + rt * TB + 2048 + (2 * j + 1) * 128 + lane * 4);
      const uint32_t wv[4] = {qw.x, qw.y, qw.z, qw.w};
      const uint32_t hws[2] = {hw0, hw1};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ksl = 4 * j + i;
        const uint32_t hw = hws[i >> 1];
        const int ip = i & 1;
        uint32_t a[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t base = lop3_and_or(wv[i] >> (4 * jj), 0x000F000Fu, 0x64006400u);
          a[jj] = lop3_or_and(base, shift_signed(hw, 2 * (4 * ip + jj) - 4), 0x00300030u);
        }
        const float2 sc = *reinterpret_cast<const float2*>(scr + ((rt * 16 + ksl) * 8 + g) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float d[4];
          const float c0 = xsum[i][nt].x, c1 = xsum[i][nt].y;  // already -1056 x the sums
          mma_f16(d, a[0], a[1], a[2], a[3], bq[i][nt][0], bq[i][nt][1], c0, c1, c0, c1);
          float* ac = acc[rt][nt];
          ac[0] = fmaf(sc.x, d[0], ac[0]);
          ac[1] = fmaf(sc.x, d[1], ac[1]);
          ac[2] = fmaf(sc.y, d[2], ac[2]);
          ac[3] = fmaf(sc.y, d[3], ac[3]);
        }
      }
    }
  }
}

template <int NT>
SPEC_DEV void tile_q80(const uint8_t* tp, const uint8_t* xs, const float* scr, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 2176;
  const int g = lane >> 2;
  const uint8_t* x32 = xs + 8 * NT * 256;
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // one Q8_0 block (32 columns) per j
    uint32_t bq[2][NT][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) load_bfrag<NT>(xs, 2 * j + i, lane, bq[i]);
    float2 xsum[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xsum[nt] = load_sum<NT>(x32, j, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const float2 sc = *reinterpret_cast<const float2*>(scr + ((rt * 4 + j) * 8 + g) * 2);
      const uint32_t w[4] = {qw.x ^ 0x80808080u, qw.y ^ 0x80808080u, qw.z ^ 0x80808080u, qw.w ^ 0x80808080u};
      uint32_t a[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        a[h][0] = __byte_perm(w[2 * h], 0x64646464u, 0x4140);
        a[h][1] = __byte_perm(w[2 * h], 0x64646464u, 0x4342);
        a[h][2] = __byte_perm(w[2 * h + 1], 0x64646464u, 0x4140);
        a[h][3] = __byte_perm(w[2 * h + 1], 0x64646464u, 0x4342);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float d[4];
        // -1152 x the sums = 1.125 x the stored -1024 x the sums (one rounding, as before)
        const float c0 = 1.125f * xsum[nt].x, c1 = 1.125f * xsum[nt].y;
        mma_f16(d, a[0][0], a[0][1], a[0][2], a[0][3], bq[0][nt][0], bq[0][nt][1], c0, c1, c0, c1);
        mma_f16(d, a[1][0], a[1][1], a[1][2], a[1][3], bq[1][nt][0], bq[1][nt][1], d[0], d[1], d[2], d[3]);
        float* ac = acc[rt][nt];
        ac[0] = fmaf(sc.x, d[0], ac[0]);
        ac[1] = fmaf(sc.x, d[1], ac[1]);
        ac[2] = fmaf(sc.y, d[2], ac[2]);
        ac[3] = fmaf(sc.y, d[3], ac[3]);
      }
    }
  }
}

// BF16 weights never come here: they run on the tcgen05 path of fwd_kernel.
template <int F, int NT>
SPEC_DEV void process_tile(const uint8_t* tp, const uint8_t* xs, float* scr, int lane, float (&acc)[2][NT][4]) {
  decode_scales<F>(tp, scr, lane);
  __syncwarp();
  if constexpr (F == WF_Q4_K) tile_q45k<NT>(tp, xs, scr, lane, false, acc);
  else if constexpr (F == WF_Q5_K) tile_q45k<NT>(tp, xs, scr, lane, true, acc);
  else if constexpr (F == WF_Q6_K) tile_q6k<NT>(tp, xs, scr, lane, acc);
  else if constexpr (F == WF_Q8_0) tile_q80<NT>(tp, xs, scr, lane, acc);
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Operand-fragment writer used by the producing epilogues.
// ---------------------------------------------------------------------------
SPEC_DEV void frag_store(uint32_t* frag, int nt_total, int m, int k, uint16_t bits, int bf16) {
  reinterpret_cast<uint16_t*>(frag)[operand_half_index(nt_total, m, k, bf16 != 0)] = bits;
}

SPEC_DEV uint16_t round_act(float v, int bf16, float& back) {
  if (bf16) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    back = __bfloat162float(b);
    return __bfloat16_as_ushort(b);
  }
  const __half h = __float2half_rn(v);
  back = __half2float(h);
  return __half_as_ushort(h);
}

// Writes the values v[0..3] of row m at columns k0 .. k0 + 3 of the next
// operand (one 8-byte or two 4-byte stores) and the per-16 / per-32 column
// sums of the rounded values.  Called by a full warp: every lane owns 4
// consecutive columns (k0 a multiple of 4), lanes 4i .. 4i + 3 one aligned
// 16-column run; lanes with ok == false store nothing but take part in the
// shuffles.
SPEC_DEV void emit_operand4(uint32_t* frag, float* xs16, float* xs32, int nt_total, int m, int k0, const float (&v)[4],
                            int bf16, int lane, bool ok) {
  float back[4];
  uint16_t b[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) b[e] = round_act(v[e], bf16, back[e]);
  if (ok) {
    const uint32_t lo = (uint32_t)b[0] | ((uint32_t)b[1] << 16), hi = (uint32_t)b[2] | ((uint32_t)b[3] << 16);
    uint16_t* hp = reinterpret_cast<uint16_t*>(frag);
    if (bf16) {
      *reinterpret_cast<uint2*>(hp + operand_half_index(nt_total, m, k0, true)) = make_uint2(lo, hi);
    } else {
      *reinterpret_cast<uint32_t*>(hp + operand_half_index(nt_total, m, k0, false)) = lo;
      *reinterpret_cast<uint32_t*>(hp + operand_half_index(nt_total, m, k0 + 2, false)) = hi;
    }
  }
  float s16 = ((back[0] + back[1]) + back[2]) + back[3];
  s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
  s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
  const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 4);
  if (ok) {
    const int w16 = 8 * nt_total;
    if ((lane & 3) == 0) xs16[(size_t)(k0 >> 4) * w16 + m] = kXSum16Seed * s16;
    if ((lane & 7) == 0) xs32[(size_t)(k0 >> 5) * w16 + m] = kXSum32Seed * s32;
  }
}

// ---------------------------------------------------------------------------
// Split-K reduction and fused epilogues.
// ---------------------------------------------------------------------------
// Barrier among the 128 consumer threads only (the producer warp runs ahead).
SPEC_DEV void consumer_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Arrival on a split counter: release (this CTA's partial stores, ordered
// before it by the preceding barrier) and acquire (the other pieces'
// partials, for the CTA that arrives last).
SPEC_DEV int atom_add_acq_rel(int* ptr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
  return old;
}
// Completion count of an op: release of this CTA's epilogue writes.
SPEC_DEV void red_add_release(int* ptr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
// Arrival on another GPU's counter (system scope, after fence.sc.sys).
SPEC_DEV void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
SPEC_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
SPEC_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
SPEC_DEV void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
SPEC_DEV void red_add_release_sys_u64(unsigned long long* ptr, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
SPEC_DEV void st_relaxed_gpu(int* ptr, int v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
SPEC_DEV int ld_relaxed_gpu(const int* ptr) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
SPEC_DEV void red_add_relaxed(int* ptr, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
SPEC_DEV void st_relaxed_sys_u64x2(unsigned long long* ptr, unsigned long long a, unsigned long long b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(ptr), "l"(a), "l"(b) : "memory");
}
SPEC_DEV void ld_relaxed_sys_u64x2(const unsigned long long* ptr, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(ptr) : "memory");
}

// Finishes one piece (the part of a 128-row group inside one chunk).  A
// group that lies in one chunk goes straight to the fused epilogue.  A group
// cut across chunks i0..i1 leaves one partial per piece in slot (chunk +
// group); the CTA that delivers the last piece sums the slots in chunk order
// and runs the epilogue.  The CTA that ran the epilogue bumps `done`.
// UM: acc came from tensor memory (tcgen05 path): thread `lane` of warp w holds
// row 32w + lane, acc[rt][nt][i] = column (rt * NT + nt) * 4 + i; otherwise acc
// is in m16n8k16 accumulator order.  Partials are stored and summed
// position-wise, so only the final placement into ys depends on it.
template <int NT, bool UM>
SPEC_DEV void reduce_and_epilogue(const QmvParams& p, int group, int own, int i0, int i1, float (&acc)[2][NT][4],
                                  float* ys, int* done, int* gflag = nullptr, unsigned epoch = 0) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  __shared__ int s_last;
  __shared__ float s_rinv[kMaxRows];
  __shared__ float s_red[kGemvWarps][kMaxRows];
  const int M = p.M;
  const int H = p.n_rows, n0 = group * kGroupRows;
  consumer_sync();  // all warps are done with their scale scratch (aliased by ys)

  // Loads of the epilogue that do not depend on the split reduction are
  // issued (by the CTA that runs the epilogue only) before the partial sums,
  // so their latency overlaps the partial-sum round trips: the sum-of-squares
  // tables and the rows' positions / cache slots go to shared memory by
  // cp.async (no registers held), and for EPI_RESID this thread's residual
  // column (every row) and norm weight go to registers.
  // EPI_QKV's row positions / cache slots live in s_red's rows 0-1.
  int* s_pos = reinterpret_cast<int*>(&s_red[0][0]);
  int* s_slot = s_pos + kMaxRows;
  float* sst = ys + M * kGroupRows;
  const int n_ss = p.ss_groups * M;
  const float* ss_t1 = p.ss_in ? p.ss_pre : nullptr;
  const float* ss_t0 = p.ss_in ? p.ss_in : p.ss_scale;
  const bool resid_pre = p.epi == EPI_RESID;
  float4 hpre4[2 * NT];  // EPI_RESID: rows warp + 4i, columns 4 lane .. 4 lane + 3
  float4 nwpre4 = make_float4(1.f, 1.f, 1.f, 1.f);
  auto epi_loads = [&]() {
    if (ss_t0) {
      for (int i = tid; i < n_ss; i += kGemvWarps * 32) {
        const int q = i / M, m = i - q * M;
        cp_async4(sst + i, ss_t0 + q * kSsStride + m);
        if (ss_t1) cp_async4(sst + n_ss + i, ss_t1 + q * kSsStride + m);
      }
    }
    if (p.epi == EPI_QKV && tid < M) {
      cp_async4(s_pos + tid, p.positions + tid);
      cp_async4(s_slot + tid, p.kv_slots + tid);
    }
    if (resid_pre) {
      const int k0 = n0 + lane * 4;
#pragma unroll
      for (int i = 0; i < 2 * NT; ++i) {
        const int m = warp + 4 * i;
        hpre4[i] = m < M ? __ldcg(reinterpret_cast<const float4*>(p.h + (size_t)m * H + k0)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (p.next_norm) nwpre4 = __ldg(reinterpret_cast<const float4*>(p.next_norm + k0));
    }
  };
  if (i0 == i1) epi_loads();

  if (i0 != i1) {
    const size_t per = (size_t)kGroupRows * 8 * NT;
    float* mine = p.part + (size_t)(own + group) * per;
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        __stcg(reinterpret_cast<float4*>(mine + ((size_t)((warp * 2 + rt) * NT + nt) * 32 + lane) * 4),
               make_float4(acc[rt][nt][0], acc[rt][nt][1], acc[rt][nt][2], acc[rt][nt][3]));
    consumer_sync();
    if (tid == 0) {
      const int prev = atom_add_acq_rel(&p.counters[group], 1);
      s_last = (prev == i1 - i0);
      if (s_last) p.counters[group] = 0;
    }
    consumer_sync();
    if (!s_last) return;  // uniform across the CTA
    epi_loads();
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[rt][nt][i] = 0.f;
    // Sum the pieces in chunk order; the loads of SB pieces are issued together.
    constexpr int SB = NT == 1 ? 4 : (NT == 2 ? 2 : 1);
    for (int s0 = i0; s0 <= i1; s0 += SB) {
      float4 v[SB][2][NT];
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        if (s0 + q <= i1) {
          const float* ps = p.part + (size_t)(s0 + q + group) * per;
#pragma unroll
          for (int rt = 0; rt < 2; ++rt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              v[q][rt][nt] =
                  __ldcg(reinterpret_cast<const float4*>(ps + ((size_t)((warp * 2 + rt) * NT + nt) * 32 + lane) * 4));
        }
      }
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        if (s0 + q <= i1) {
#pragma unroll
          for (int rt = 0; rt < 2; ++rt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[rt][nt][0] += v[q][rt][nt].x;
              acc[rt][nt][1] += v[q][rt][nt].y;
              acc[rt][nt][2] += v[q][rt][nt].z;
              acc[rt][nt][3] += v[q][rt][nt].w;
            }
        }
      }
    }
  }
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (UM) {
          const int col = (rt * NT + nt) * 4 + i;
          if (col < M) ys[col * kGroupRows + warp * 32 + lane] = acc[rt][nt][i];
        } else {
          const int row = warp * 32 + rt * 16 + g + ((i >> 1) ? 8 : 0);
          const int col = nt * 8 + 2 * t + (i & 1);
          if (col < M) ys[col * kGroupRows + row] = acc[rt][nt][i];
        }
      }
  if (p.tp_size > 1) {
    // Tensor parallelism: this rank's sum of the group goes to every rank's
    // receive slot as flagged words (peers first, this rank last); then each
    // thread waits for its elements' words from every rank and adds them in
    // rank order (the same arithmetic on every rank, so h stays identical).
    // Each thread reads back only the elements it stored, so ys needs no
    // barrier between the two loops.
    // Two words per 16-byte store / load (each 8-byte word is read and
    // checked on its own, so a pair need not arrive together).
    consumer_sync();
    const int ng = p.seg[0].groups + p.seg[1].groups;
    const int n = M * kGroupRows;  // even
    const unsigned flag = tp_flag_of(*p.tp_epoch, p.tp_tag);
    const unsigned long long hi = (unsigned long long)flag << 32;
    for (int i = 1; i <= p.tp_size; ++i) {
      const int r = (p.tp_rank + i) % p.tp_size;
      unsigned long long* dst = p.tp_recv[r] + ((size_t)p.tp_rank * ng + group) * kTpSlot;
      for (int e = 2 * tid; e < n; e += 2 * kGemvWarps * 32)
        st_relaxed_sys_u64x2(dst + e, hi | __float_as_uint(ys[e]), hi | __float_as_uint(ys[e + 1]));
    }
    bool live = true;
    const unsigned long long t0 = global_timer_ns();
    for (int e = 2 * tid; e < n; e += 2 * kGemvWarps * 32) {
      float sum0 = 0.f, sum1 = 0.f;
      for (int r = 0; r < p.tp_size; ++r) {
        const unsigned long long* src = p.tp_recv_local + ((size_t)r * ng + group) * kTpSlot + e;
        unsigned long long w0, w1;
        ld_relaxed_sys_u64x2(src, w0, w1);
        for (unsigned spin = 0; live && ((unsigned)(w0 >> 32) != flag || (unsigned)(w1 >> 32) != flag); ++spin) {
          if ((spin & 255u) == 255u &&
              ((*(volatile unsigned*)p.err & DEV_ERR_MBAR_TIMEOUT) || global_timer_ns() - t0 > kMbarTimeoutNs)) {
            live = false;
            atomicOr(p.err, DEV_ERR_MBAR_TIMEOUT);
            if (atomicCAS(p.err + 1, 0u, WAIT_TP_PEERS | ((unsigned)group << 8) | ((unsigned)blockIdx.x << 16)) ==
                0u) {
              p.err[2] = (unsigned)r;
              p.err[3] = (unsigned)(((unsigned)(w0 >> 32) != flag ? w0 : w1) >> 32);
            }
            break;
          }
          ld_relaxed_sys_u64x2(src, w0, w1);
        }
        sum0 += __uint_as_float((unsigned)w0);
        sum1 += __uint_as_float((unsigned)w1);
      }
      ys[e] = sum0;
      ys[e + 1] = sum1;
    }
  }
  cp_async_wait_all();  // sst, s_pos, s_slot
  if (ss_t0) {
    // Per-group sums of squares of the residual rows -> RMSNorm scale: thread
    // m adds row m's groups in group order (the same order for every M, and
    // the final-norm kernel's); threads 64 + m do the pre-scale table.
    consumer_sync();
    const bool t1 = ss_t1 && tid >= kMaxRows && tid - kMaxRows < M;
    if (tid < M || t1) {
      const float* col = t1 ? sst + n_ss + (tid - kMaxRows) : sst + tid;
      float ms = 0.f;
#pragma unroll 8
      for (int q = 0; q < p.ss_groups; ++q) ms += col[q * M];
      // s_red[3] is free (s_pos / s_slot use rows 0-1).
      if (t1) s_red[3][tid - kMaxRows] = ms;
      else s_rinv[tid] = ms;
    }
    consumer_sync();
    if (tid < M) {
      float r = 1.f / sqrtf(s_rinv[tid] * p.ss_inv_dim + p.eps);
      // undo the pre-scale the operand was emitted with: x (1/r_pre) r
      if (ss_t1) r *= sqrtf(s_red[3][tid] * p.ss_inv_dim + p.eps);
      // EPI_RESID (ss_scale): s_rinv is the pre-scale of the emitted operand.
      s_rinv[tid] = r;
    }
  } else if (tid < M) {
    s_rinv[tid] = 1.f;
  }
  consumer_sync();

  if (p.epi == EPI_STORE) {
    if (p.out_peers) {
      // Vocabulary-parallel head: the rows go to every rank's logits buffer.
      float* dst[kTpMaxRanks];
      const int T = p.out_ranks < kTpMaxRanks ? p.out_ranks : kTpMaxRanks;
      for (int r = 0; r < T; ++r) dst[r] = p.out_peers[r];
      for (int idx = tid; idx < M * kGroupRows; idx += kGemvWarps * 32) {
        const int m = idx / kGroupRows, j = idx % kGroupRows, n = n0 + j;
        float v = ys[m * kGroupRows + j] * s_rinv[m];
        if (p.bias) v += p.bias[n];
        for (int r = 0; r < T; ++r) dst[r][(size_t)m * p.ld_out + n] = v;
      }
    } else {
      for (int idx = tid; idx < M * kGroupRows; idx += kGemvWarps * 32) {
        const int m = idx / kGroupRows, j = idx % kGroupRows, n = n0 + j;
        float v = ys[m * kGroupRows + j] * s_rinv[m];
        if (p.bias) v += p.bias[n];
        p.out[(size_t)m * p.ld_out + n] = v;
      }
    }
  } else if (p.epi == EPI_QKV) {
    // Thread t owns columns [j0, j0 + 8), j0 = 8 (t % 16), of rows t / 16,
    // t / 16 + 8, ...: one 16-byte store per row.  (Each 2-byte store is an
    // instruction of its own, and under the weight stream every store
    // instruction costs about a memory round trip of issue time.)
    const int hd = p.head_dim, nq = p.n_q_heads, nkv = p.n_kv_heads;
    const int G = nq / nkv, R = M * G, half = hd / 2;
    const int j0 = (tid & 15) * 8, n = n0 + j0;
    const int d0 = n % hd, head = n / hd;  // the 8 columns lie in one head (hd % 8 == 0)
    const bool is_v = head >= nq + nkv;
    const bool ilv = p.rope_interleaved != 0;
    // Partner column of column j0 + e (RoPE pairs): e ^ 1 within the block
    // (interleaved pairs), or j0 + e -/+ half (rotate-half); table column of
    // the block's first pair.
    const int jq = ilv ? j0 : (d0 < half ? j0 + half : j0 - half);
    const int ci0 = ilv ? (d0 >> 1) : (d0 < half ? d0 : d0 - half);
    const bool lowhalf = d0 < half;
    float bx[8], by[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      bx[e] = p.bias ? p.bias[n + e] : 0.f;
      by[e] = (p.bias && !is_v) ? p.bias[n0 + (ilv ? (j0 + (e ^ 1)) : (jq + e))] : 0.f;
    }
    uint16_t* dst;
    size_t stride_m;  // per row m: q rows move by G * hd; cache rows by the slot
    if (head < nq) {
      const int kvh = head / G, gq = head % G;
      dst = reinterpret_cast<uint16_t*>(p.qbuf) + ((size_t)kvh * R + gq) * hd + d0;
      stride_m = (size_t)G * hd;
    } else if (!is_v) {
      dst = reinterpret_cast<uint16_t*>(p.kcache) + (size_t)(head - nq) * p.t_max * hd + d0;
      stride_m = 0;
    } else {
      dst = reinterpret_cast<uint16_t*>(p.vcache) + (size_t)(head - nq - nkv) * p.t_max * hd + d0;
      stride_m = 0;
    }
    for (int m = tid >> 4; m < M; m += 8) {
      const float rinv = s_rinv[m];
      float x[8], y[8], cs[8], sn[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        x[e] = ys[m * kGroupRows + j0 + e] * rinv;
        if (p.bias) x[e] += bx[e];
        cs[e] = 1.f;
        sn[e] = 0.f;
        y[e] = 0.f;
      }
      if (!is_v) {
        const size_t tb = (size_t)s_pos[m] * half + ci0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          y[e] = ys[m * kGroupRows + (ilv ? j0 + (e ^ 1) : jq + e)] * rinv;
          if (p.bias) y[e] += by[e];
          const size_t ti = tb + (ilv ? (e >> 1) : e);
          cs[e] = p.rope_cos[ti];
          sn[e] = p.rope_sin[ti];
        }
      }
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float o2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int ee = e + h;
          const bool first = ilv ? ((ee & 1) == 0) : lowhalf;
          o2[h] = is_v ? x[ee] : (first ? (x[ee] * cs[ee] - y[ee] * sn[ee]) : (y[ee] * sn[ee] + x[ee] * cs[ee]));
        }
        float back;
        w[e >> 1] = (uint32_t)round_act(o2[0], p.act_bf16, back) | ((uint32_t)round_act(o2[1], p.act_bf16, back) << 16);
      }
      *reinterpret_cast<uint4*>(dst + (stride_m ? (size_t)m * stride_m : (size_t)s_slot[m] * hd)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else if (p.epi == EPI_RESID) {
    // Warp w owns rows w, w + 4, ...; lane l owns columns [4l, 4l + 4) of the
    // group: float4 residual updates (rows loaded before the partial sums), a
    // row's sum of squares in one warp reduction, 4 operand values per store.
    // s_rinv[m] = rinv of the residual before this update (or 1).
    const int k0 = n0 + lane * 4;
    const float4 nw = nwpre4;  // 1 without a next norm
#pragma unroll
    for (int i = 0; i < 2 * NT; ++i) {
      const int m = warp + 4 * i;
      if (m < M) {  // uniform across the warp
        const float4 y = *reinterpret_cast<const float4*>(ys + m * kGroupRows + lane * 4);
        float4 hv = hpre4[i];
        hv.x += y.x;
        hv.y += y.y;
        hv.z += y.z;
        hv.w += y.w;
        *reinterpret_cast<float4*>(p.h + (size_t)m * H + k0) = hv;
        const float sq = warp_sum(((hv.x * hv.x + hv.y * hv.y) + hv.z * hv.z) + hv.w * hv.w);
        if (lane == 0) p.ss_out[group * kSsStride + m] = sq;
        if (p.next_frag) {
          const float r = s_rinv[m];
          const float v[4] = {hv.x * nw.x * r, hv.y * nw.y * r, hv.z * nw.z * r, hv.w * nw.w * r};
          emit_operand4(p.next_frag, p.next_xsum16, p.next_xsum32, NT, m, k0, v, p.act_bf16, lane, true);
        }
      }
    }
  } else if (p.epi == EPI_SILU) {
    // Thread t owns gate/up columns [4c, 4c + 4) (c = t % 16) of rows t / 16,
    // t / 16 + 8, ...: 4 operand values per store.
    const int c = (tid & 15) * 4, f0 = p.next_col_off + group * 64 + c;
    for (int mb = 0; mb < M; mb += 8) {  // uniform across the CTA
      const int m = mb + (tid >> 4);
      const bool ok = m < M;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok) {
        const float r = s_rinv[m];
        const float4 g4 = *reinterpret_cast<const float4*>(ys + m * kGroupRows + c);
        const float4 u4 = *reinterpret_cast<const float4*>(ys + m * kGroupRows + 64 + c);
        const float gv[4] = {g4.x * r, g4.y * r, g4.z * r, g4.w * r};
        const float uv[4] = {u4.x * r, u4.y * r, u4.z * r, u4.w * r};
#pragma unroll
        for (int e = 0; e < 4; ++e) a[e] = gv[e] / (1.f + expf(-gv[e])) * uv[e];
      }
      emit_operand4(p.next_frag, p.next_xsum16, p.next_xsum32, NT, ok ? m : 0, f0, a, p.act_bf16, lane, ok);
    }
  }
  consumer_sync();  // ys aliases the scale scratch of the next unit
  if (p.out_counters && tid == 0) {
    // Every thread's peer stores are ordered before this by the barrier; the
    // system-scope fence makes them visible to the other GPUs before the
    // arrivals they wait on.
    fence_acq_rel_sys();
    const int T = p.out_ranks < kTpMaxRanks ? p.out_ranks : kTpMaxRanks;
    for (int r = 0; r < T; ++r) red_add_release_sys_u64(p.out_counters[r], 1ull);
  }
  if (done && tid == 0) {
    if (gflag) {  // one release fence covers the group flag and the op count
      fence_acq_rel_gpu();
      st_relaxed_gpu(gflag + group, (int)epoch);
      red_add_relaxed(done, 1);
    } else {
      red_add_release(done, 1);
    }
  }
}

SPEC_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

constexpr int kProducerWarp = kGemvWarps;  // warp 4
constexpr int kMmaWarp = kGemvWarps + 1;    // warp 5 (tcgen05 path only): issues the MMAs
constexpr int kStageBudget = 64 * 1024;    // ring bytes per CTA (3 CTAs / SM at M <= 8)
constexpr int kUmmaSmemBudget = 215 * 1024;  // dynamic shared memory of a tcgen05 CTA (one per SM)

template <int SET, int F, int NT>
struct GeoIf {
  static constexpr bool on = (SET & fmt_bit(F)) != 0;
  static constexpr int PAIR = on ? Geo<F, NT>::PAIR : 0;
  static constexpr int XB = on ? Geo<F, NT>::XB : 0;
};
constexpr int cmax(int a, int b) { return a > b ? a : b; }

template <int SET, int NT>
struct FGeo {
  static constexpr int PAIRMAX =
      cmax(cmax(cmax(GeoIf<SET, WF_Q4_K, NT>::PAIR, GeoIf<SET, WF_Q5_K, NT>::PAIR),
                cmax(GeoIf<SET, WF_Q6_K, NT>::PAIR, GeoIf<SET, WF_Q8_0, NT>::PAIR)),
           GeoIf<SET, WF_BF16, NT>::PAIR);
  static constexpr int XBMAX = cmax(cmax(cmax(GeoIf<SET, WF_Q4_K, NT>::XB, GeoIf<SET, WF_Q5_K, NT>::XB),
                                         cmax(GeoIf<SET, WF_Q6_K, NT>::XB, GeoIf<SET, WF_Q8_0, NT>::XB)),
                                    GeoIf<SET, WF_BF16, NT>::XB);
  // BF16 (the only format of its set) runs on tcgen05: one CTA per SM, whose
  // MMAs are issued by one thread, so the ring takes most of shared memory.
  static constexpr bool UM = SET == FS_BF16;
  static constexpr int STAGE = kGemvWarps * PAIRMAX + XBMAX;
  static constexpr int SCR = kGemvWarps * kScratch;
  static constexpr int YS = (8 * NT * kGroupRows + 2 * kMaxSsGroups * 8 * NT) * 4;
  static constexpr int TAIL = SCR > YS ? SCR : YS;
  static constexpr int D0 = (UM ? kUmmaSmemBudget - TAIL : kStageBudget) / STAGE;
  static constexpr int D = D0 < 2 ? 2 : (D0 > 6 ? 6 : D0);
  static constexpr int RING = D * STAGE;
  static constexpr int SMEM = RING + TAIL;
  // tcgen05 MMA shape: M = 128 rows of a group, N = the operand's rows
  // (at least 16; one n-tile is read twice through a zero row-group stride).
  // Two accumulators in TMEM: the MMAs of one piece run while the consumer
  // warps drain the previous one.
  static constexpr int UN = NT < 2 ? 16 : 8 * NT;
  static constexpr uint32_t TCOLS = 2 * UN <= 32 ? 32u : (uint32_t)(2 * UN);  // TMEM columns allocated
  static constexpr int THREADS = (kGemvWarps + (UM ? 2 : 1)) * 32;
};

// Stage s of an op: segment, group (within the segment and overall), k-tile.
struct StageLoc {
  int seg, lgrp, grp, kt, gstart;  // gstart: stage index of the group's first k-tile
};
SPEC_DEV StageLoc locate(const QmvParams& q, int s) {
  StageLoc L;
  const int a = q.seg[0].groups * q.seg[0].k_tiles;
  L.seg = s < a ? 0 : 1;
  const int r = L.seg ? s - a : s;
  const int kt = q.seg[L.seg].k_tiles;
  L.lgrp = r / kt;
  L.kt = r - L.lgrp * kt;
  L.grp = (L.seg ? q.seg[0].groups : 0) + L.lgrp;
  L.gstart = s - L.kt;
  return L;
}
SPEC_DEV int chunk_start(const QmvParams& q, int i) { return (int)(((long long)i * q.stages) / q.chunks); }
// Chunk holding stage s: the largest i with chunk_start(i) <= s.
SPEC_DEV int chunk_of(const QmvParams& q, int s) { return (int)(((long long)(s + 1) * q.chunks - 1) / q.stages); }

// Walks (op, chunk, stage) for CTA c in schedule order: chunks c, c+G, ...
// The producer's walks skip the attention ops (no weight stream).
// A GEMV chunk [s0, s_end) that starts inside a group and reaches the next
// group's start b is walked [b, s_end) then [s0, b) (FwdParams::rotate): the
// piece that ends the first group -- the one whose CTA most likely arrives
// last and runs the group's reduction and epilogue -- comes after this
// CTA's other pieces of the op, so that epilogue delays none of them.  Each
// piece's own stages stay in order, so no sum changes.
struct SeqIt {
  int op = 0, k = 0, s = 0, s_end = 0;
  int s0 = 0, b = 0, v = 0, len = 0;  // chunk start, walk start, position in the walk, chunk length
  bool valid = false;
  bool gemv_only = false;
};
// Stage at position v of the chunk's walk.
SPEC_DEV int seq_stage(const SeqIt& it, int v) {
  const int l1 = it.s_end - it.b;
  return v < l1 ? it.b + v : it.s0 + (v - l1);
}

SPEC_DEV void seq_settle(const FwdParams& P, int c, int G, SeqIt& it) {
  // Move to the first non-empty chunk at or after (it.op, it.k).
  while (it.op < P.n_ops) {
    if (it.gemv_only && P.ops[it.op].kind != OPK_GEMV) {
      ++it.op;
      it.k = 0;
      continue;
    }
    const QmvParams& q = P.ops[it.op].q;
    const int i = c + it.k * G;
    if (i < q.chunks) {
      it.s0 = chunk_start(q, i);
      it.s_end = chunk_start(q, i + 1);
      if (it.s0 < it.s_end) {
        it.b = it.s0;
        if (P.rotate && P.ops[it.op].kind == OPK_GEMV) {
          const StageLoc L = locate(q, it.s0);
          const int nb = L.gstart + q.seg[L.seg].k_tiles;  // the next group's first stage
          if (L.kt != 0 && nb < it.s_end) it.b = nb;
        }
        it.v = 0;
        it.len = it.s_end - it.s0;
        it.s = seq_stage(it, 0);
        it.valid = true;
        return;
      }
      ++it.k;
      continue;
    }
    ++it.op;
    it.k = 0;
  }
  it.valid = false;
}
SPEC_DEV void seq_begin(const FwdParams& P, int c, int G, SeqIt& it, bool gemv_only) {
  it = SeqIt{};
  it.gemv_only = gemv_only;
  seq_settle(P, c, G, it);
}
SPEC_DEV void seq_next(const FwdParams& P, int c, int G, SeqIt& it) {
  if (++it.v < it.len) {
    it.s = seq_stage(it, it.v);
    return;
  }
  ++it.k;
  seq_settle(P, c, G, it);
}
// Moves past the rest of the current chunk.
SPEC_DEV void seq_next_chunk(const FwdParams& P, int c, int G, SeqIt& it) {
  it.v = it.len - 1;
  seq_next(P, c, G, it);
}

SPEC_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Records where a bounded wait gave up (first one wins), then flags it.
SPEC_DEV void wait_gave_up(unsigned* err, unsigned site, int op, int where, int seen) {
  if (atomicCAS(err + 1, 0u, site | ((unsigned)op << 8) | ((unsigned)blockIdx.x << 16)) == 0u) {
    err[2] = (unsigned)where;
    err[3] = (unsigned)seen;
  }
  atomicOr(err, DEV_ERR_MBAR_TIMEOUT);
}

SPEC_DEV int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SPEC_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

template <int SET, int NT>
SPEC_DEV void process_any(int fmt, const uint8_t* tp, const uint8_t* xs, float* scr, int lane,
                          float (&acc)[2][NT][4]) {
  if constexpr ((SET & FS_Q4K) != 0) {
    if (fmt == WF_Q4_K) return process_tile<WF_Q4_K, NT>(tp, xs, scr, lane, acc);
  }
  if constexpr ((SET & FS_Q6K) != 0) {
    if (fmt == WF_Q6_K) return process_tile<WF_Q6_K, NT>(tp, xs, scr, lane, acc);
  }
  if constexpr ((SET & FS_Q5K) != 0) {
    if (fmt == WF_Q5_K) return process_tile<WF_Q5_K, NT>(tp, xs, scr, lane, acc);
  }
  if constexpr ((SET & FS_Q80) != 0) {
    if (fmt == WF_Q8_0) return process_tile<WF_Q8_0, NT>(tp, xs, scr, lane, acc);
  }
}

SPEC_DEV int x32_bytes(int fmt, int NT) { return fmt == WF_BF16 ? 0 : (fmt_kt(fmt) / 32) * 8 * NT * 4; }
SPEC_DEV int x16_bytes(int fmt, int NT) { return fmt == WF_BF16 ? 0 : (fmt_kt(fmt) / 16) * 8 * NT * 4; }

constexpr int kAttnParamBytes = 256;  // ring bytes an attention unit keeps its parameters in
static_assert(sizeof(AttnParams) <= kAttnParamBytes, "AttnParams outgrew its ring slot");

// Keys per pass an attention split unit stages in a ring of `ring` bytes
// (a multiple of attn::kKeyBlock, at most the split's chunk).
__host__ __device__ inline int attn_keys_per_pass(int ring, int hd, int chunk) {
  const int kp = ((ring / (2 * (hd + 8)) - attn::kWarps * 16) / 2) & ~(attn::kKeyBlock - 1);
  return kp < chunk ? kp : chunk;
}

// One unit of an attention op, run by the 4 consumer warps after every GEMV
// stage of this CTA was consumed (the ring is drained and reused as the
// key / query staging).  Split units wait for the QKV groups of their KV
// head (per-group flags, or the dependency's done count) and count
// themselves in `done`; combine units wait for every split unit.
template <int NT>
SPEC_DEV void attn_op_unit(const FwdOp* ops, int* done, const int* gflags, int flag_stride, unsigned* err, int op,
                           int u, uint8_t* ring, int ring_bytes, unsigned epoch) {
  const FwdOp& fo = ops[op];
  const QmvParams& q = fo.q;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The unit's parameters live in the last bytes of the ring (shared
  // memory), not in registers.
  ring_bytes -= kAttnParamBytes;
  AttnParams* ap = reinterpret_cast<AttnParams*>(ring + ring_bytes);
  consumer_sync();  // every warp is done with the ring (GEMV stages or the previous unit)
  if (tid == 0) {
    AttnParams& a = *ap;
    a.q = q.qbuf;
    a.kcache = q.kcache;
    a.vcache = q.vcache;
    a.n_kv = q.n_kv_heads;
    a.G = q.n_q_heads / q.n_kv_heads;
    a.hd = q.head_dim;
    a.M = q.M;
    a.t_max = q.t_max;
    a.step = q.attn_step;
    a.anc = q.attn_anc;
    a.scale_log2 = q.attn_scale_log2;
    a.chunk = q.attn_chunk;
    a.max_splits = q.attn_max_splits;
    a.part_o = q.attn_o;
    a.part_ml = q.attn_ml;
    a.frag = q.next_frag;
    a.xsum16 = q.next_xsum16;
    a.xsum32 = q.next_xsum32;
    a.col_off = q.next_col_off;
    a.act_bf16 = q.act_bf16;
    a.err = q.err;
  }
  consumer_sync();
  const AttnParams& a = *ap;
  const int dep = fo.dep;
  if (fo.kind == OPK_ATTN_SPLIT) {
    const int kvh = u % a.n_kv, split = u / a.n_kv;
    auto wait_inputs = [&]() {
      if (dep >= 0 && tid == 0) {
        // The QKV groups holding this KV head's q rows, k rows and v rows.
        const int hd = a.hd, G = a.G, nq = q.n_q_heads, nkv = a.n_kv;
        const int r0[3] = {kvh * G * hd, nq * hd + kvh * hd, (nq + nkv) * hd + kvh * hd};
        const int rn[3] = {G * hd, hd, hd};
        const QmvParams& d = ops[dep].q;
        const int dgroups = d.seg[0].groups + d.seg[1].groups;
        const int* fl = gflags ? gflags + (size_t)dep * flag_stride : nullptr;
        unsigned long long t0 = 0;
        for (;;) {
          bool ok = ld_relaxed_gpu(done + dep) >= dgroups;
          if (!ok && fl) {
            ok = true;
            for (int j = 0; j < 3; ++j)
              for (int g2 = r0[j] / kGroupRows; g2 <= (r0[j] + rn[j] - 1) / kGroupRows; ++g2)
                ok &= ld_relaxed_gpu(fl + g2) == (int)epoch;
          }
          if (ok) break;
          const unsigned long long now = global_timer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kMbarTimeoutNs) {
            wait_gave_up(err, WAIT_ATTN_DEP, op, u, ld_relaxed_gpu(done + dep));
            break;
          }
        }
        fence_acq_rel_gpu();
      }
      consumer_sync();
    };
    const int kp = attn_keys_per_pass(ring_bytes, a.hd, a.chunk);
    if (a.hd == 128) {
      if (a.act_bf16) attn::split_unit<128, true, 2>(a, split, kvh, ring, kp, wait_inputs);
      else attn::split_unit<128, false, 2>(a, split, kvh, ring, kp, wait_inputs);
    } else {
      if (a.act_bf16) attn::split_unit<64, true, 2>(a, split, kvh, ring, kp, wait_inputs);
      else attn::split_unit<64, false, 2>(a, split, kvh, ring, kp, wait_inputs);
    }
    consumer_sync();  // every thread's partial stores are issued
    if (tid == 0) {
      fence_acq_rel_gpu();
      red_add_relaxed(done + op, 1);
    }
  } else {
    if (dep >= 0) {
      const int need = ops[dep].q.chunks;  // every split unit
      unsigned long long t0 = 0;
      while (ld_acquire(done + dep) < need) {
        const unsigned long long now = global_timer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kMbarTimeoutNs) {
          if (lane == 0) wait_gave_up(err, WAIT_ATTN_DEP, op, u, ld_relaxed_gpu(done + dep));
          break;
        }
      }
    }
    __syncwarp();
    if (a.hd == 128) attn::combine_item<128>(a, NT, u * kGemvWarps + warp, lane);
    else attn::combine_item<64>(a, NT, u * kGemvWarps + warp, lane);
  }
}

// CTA c takes chunks c, c + G, ... of every op.  A stage of a later op waits
// for groups that other CTAs of the launch produce, so a multi-op launch needs
// every CTA resident at once: it is launched cooperative (FwdParams::
// cooperative), which the hardware guarantees or refuses.
//
// Persistent, warp-specialized multi-op GEMV (see FwdOp).  Warp 4 lane 0 is
// the producer: it keeps a weight cursor up to D stages ahead of the
// consumers (never blocked by op dependencies) and an operand cursor that
// fills each stage's activation tile once that stage's op has its inputs.
// Warps 0-3 consume stages, run the per-unit split-K epilogue and publish
// op completion.
//
// BF16 weights (SET == FS_BF16) run on the 5th-generation tensor core
// instead: warp 5 lane 0 issues, per stage, the tcgen05.mma of the group's
// 128 rows x the operand's rows over the stage's 128 columns (8 K-steps of
// 16) into one of two TMEM accumulators, and its tcgen05.commit frees the
// ring slot once the MMAs have read it.  At the end of a piece it commits the
// accumulator to the consumer warps, which read their 32 rows (TMEM lanes)
// with tcgen05.ld, hand the accumulator back and run the same split-K
// reduction and epilogues while the next piece's MMAs proceed.
template <int SET, int NT>
__global__ void __launch_bounds__(FGeo<SET, NT>::THREADS,
                                  SET == FS_BF16 ? 1 : (NT == 1 ? 3 : (NT == 2 ? 3 : (NT == 4 ? 2 : 1))))
    fwd_kernel(const __grid_constant__ FwdParams Pg) {
  using FG = FGeo<SET, NT>;
  constexpr int D = FG::D;
  constexpr bool UM = FG::UM;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[D];
  __shared__ __align__(8) uint64_t empty[D];
  __shared__ __align__(8) uint64_t accfull[2];   // tcgen05 path: a piece's MMAs are complete
  __shared__ __align__(8) uint64_t accempty[2];  // tcgen05 path: the consumers have read the accumulator
  __shared__ __align__(8) uint64_t issdone;      // tcgen05 path: every MMA the issuer started is complete
  __shared__ uint32_t s_tmem;                    // tcgen05 path: TMEM base address
  __shared__ __align__(16) FwdOp s_ops[kMaxLaunchOps];
  // Dependent launch.  Without a cooperative launch the kernels after this
  // one (attention, then the next forward kernel) are only scheduled as its
  // CTAs exit: letting them launch early let CTAs of the next forward kernel
  // become resident before their siblings and wait on them, and a split-K
  // group's completion was lost on B200 (a bounded wait fired).  When the
  // forward kernels are cooperative that cannot happen (the next one starts
  // only when all of its CTAs fit), so they trigger at entry: the attention
  // CTAs take the slots of exiting CTAs at once and stage the older keys
  // while this launch's tail finishes.
  if (Pg.trigger_at_start) pdl_launch_dependents();
  // Op descriptors live in shared memory for the whole launch (the producer
  // walks them per tile).  They were uploaded long before this launch.
  {
    const int n = Pg.n_ops < kMaxLaunchOps ? Pg.n_ops : kMaxLaunchOps;
    const int4* src = reinterpret_cast<const int4*>(Pg.ops);
    int4* dst = reinterpret_cast<int4*>(s_ops);
    const int words = n * (int)(sizeof(FwdOp) / sizeof(int4));
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  FwdParams P = Pg;
  P.ops = s_ops;
  // This forward's number (the host writes it before the first kernel of
  // the forward; it does not change while the forward runs).
  const unsigned epoch = P.epoch ? *P.epoch : 0u;
  uint8_t* ring = smem;
  float* tail = reinterpret_cast<float*>(smem + FG::RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < D; ++s) {
      mbar_init(&full[s], 1);
      // tcgen05 path: the slot is freed by the one commit after its MMAs.
      mbar_init(&empty[s], UM ? 1 : kGemvWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], kGemvWarps);
    }
    mbar_init(&issdone, 1);
  }
  fence_mbar_init();
  if constexpr (UM) {
    if (warp == 0) tmem_alloc(&s_tmem, FG::TCOLS);
    tc_fence_before();
  }
  __syncthreads();
  if constexpr (UM) tc_fence_after();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // Weights are read once per forward: evict them from L2 first.
      const uint64_t wpol = l2_policy_evict_first();
      auto issue_w = [&](const SeqIt& it, int pos) {
        const QmvParams& q = P.ops[it.op].q;
        const StageLoc L = locate(q, it.s);
        const WSeg& sg = q.seg[L.seg];
        const int fmt = sg.fmt, pair = fmt_pair_bytes(fmt);
        const int xb = (fmt_kt(fmt) / 16) * NT * 256 + x32_bytes(fmt, NT) + x16_bytes(fmt, NT);
        const int st = pos % D;
        mbar_arrive_expect_tx(&full[st], kGemvWarps * pair + xb);
        uint8_t* dst = ring + (size_t)st * FG::STAGE;
        // The stage's 4 pair tiles are contiguous in HBM: one bulk copy.
        tma_bulk_g2s_hint(dst, sg.w + ((size_t)L.lgrp * sg.k_tiles + L.kt) * kGemvWarps * pair, kGemvWarps * pair,
                          &full[st], wpol);
      };
      auto issue_x = [&](const SeqIt& it, int pos) {
        const QmvParams& q = P.ops[it.op].q;
        const StageLoc L = locate(q, it.s);
        const int fmt = q.seg[L.seg].fmt;
        const int ksf = fmt_kt(fmt) / 16;
        const int ks0 = L.kt * ksf;
        const int xf = ksf * NT * 256, x32 = x32_bytes(fmt, NT), x16 = x16_bytes(fmt, NT);
        const int st = pos % D;
        uint8_t* dst = ring + (size_t)st * FG::STAGE + kGemvWarps * FG::PAIRMAX;
        tma_bulk_g2s(dst, reinterpret_cast<const uint8_t*>(q.xfrag) + (size_t)ks0 * NT * 256, xf, &full[st]);
        if (x32) tma_bulk_g2s(dst + xf, q.xsum32 + (size_t)(ks0 / 2) * 8 * NT, x32, &full[st]);
        if (x16) tma_bulk_g2s(dst + xf + x32, q.xsum16 + (size_t)ks0 * 8 * NT, x16, &full[st]);
      };
      // L2 run-ahead: stage `pi` of this CTA's weight stream is prefetched
      // into L2 while the ring is still `l2_ahead` stages behind, so HBM keeps
      // streaming while ops wait on their inputs (and before pdl_wait, while
      // the previous kernel still runs).
      auto issue_pf = [&](const SeqIt& it) {
        const QmvParams& q = P.ops[it.op].q;
        const StageLoc L = locate(q, it.s);
        const WSeg& sg = q.seg[L.seg];
        const int pair = fmt_pair_bytes(sg.fmt);
        tma_prefetch_l2(sg.w + ((size_t)L.lgrp * sg.k_tiles + L.kt) * kGemvWarps * pair, kGemvWarps * pair);
      };
      SeqIt wi, xi, pi;
      seq_begin(P, c, G, wi, true);
      xi = wi;
      pi = wi;
      int wpos = 0, xpos = 0, ppos = 0;
      const int ahead = P.l2_ahead;
      for (; pi.valid && ppos < D + ahead; ++ppos) {
        if (ppos >= D) issue_pf(pi);
        seq_next(P, c, G, pi);
      }
      for (; wi.valid && wpos < D; ++wpos) {  // weights only depend on nothing
        issue_w(wi, wpos);
        seq_next(P, c, G, wi);
      }
      pdl_wait();  // operands and counters come from the previous kernel
      int ready_op = -1;
      // Stage readiness with per-group flags: the groups of the dependency
      // that produce this stage's K range (128 output rows per group, 64
      // activations per group after the SiLU epilogue) must carry this
      // forward's epoch.  The dependency's `done` count is read alongside;
      // once it is full, the rest of the op needs no more checks.
      auto stage_ready = [&](const SeqIt& it) -> bool {
        const int dep = P.ops[it.op].dep;
        if (dep < 0) return true;
        const QmvParams& d = P.ops[dep].q;
        const int dgroups = d.seg[0].groups + d.seg[1].groups;
        if (!P.gflags) return ld_acquire(P.done + dep) >= dgroups;
        const QmvParams& q = P.ops[it.op].q;
        const StageLoc L = locate(q, it.s);
        const int KT = fmt_kt(q.seg[L.seg].fmt);
        const int cpg = d.epi == EPI_SILU ? kGroupRows / 2 : kGroupRows;
        const int g0 = (L.kt * KT) / cpg, g1 = (L.kt * KT + KT - 1) / cpg;
        const int* fl = P.gflags + (size_t)dep * P.flag_stride;
        const int all = ld_relaxed_gpu(P.done + dep);
        bool ok = true;
        for (int g = g0; g <= g1; ++g) ok &= ld_relaxed_gpu(fl + g) == (int)epoch;
        if (all >= dgroups) {
          ok = true;
          ready_op = it.op;
        }
        if (ok) fence_acq_rel_gpu();
        return ok;
      };
      unsigned long long t_idle = 0;
      while (xi.valid) {
        bool progressed = false;
        if (xpos < wpos) {
          if (xi.op <= ready_op || stage_ready(xi)) {
            fence_proxy_async_global();
            issue_x(xi, xpos);
            seq_next(P, c, G, xi);
            ++xpos;
            progressed = true;
          }
        }
        if (wi.valid && mbar_test_wait(&empty[wpos % D], (uint32_t)(((wpos / D) - 1) & 1))) {
          issue_w(wi, wpos);
          seq_next(P, c, G, wi);
          ++wpos;
          progressed = true;
          if (pi.valid && ppos < wpos + D + ahead) {
            issue_pf(pi);
            seq_next(P, c, G, pi);
            ++ppos;
          }
        }
        if (progressed) {
          t_idle = 0;
        } else {
          const unsigned long long now = global_timer_ns();
          if (t_idle == 0) t_idle = now;
          else if (now - t_idle > kMbarTimeoutNs) {
            const int dep = P.ops[xi.op].dep;
            wait_gave_up(P.err, WAIT_PRODUCER_IDLE, xi.op, xpos | (wpos << 16), dep >= 0 ? ld_acquire(P.done + dep) : -1);
            break;
          }
        }
      }
      // Every issued copy must land before this CTA can retire.
      const int first = wpos > D ? wpos - D : 0;
      for (int pos = first; pos < wpos; ++pos)
        if (!mbar_wait_bounded(&full[pos % D], (uint32_t)((pos / D) & 1), nullptr))
          wait_gave_up(P.err, WAIT_PRODUCER_DRAIN, xi.valid ? xi.op : 255, pos, wpos);
    }
    return;
  }

  if constexpr (UM) {
    if (warp == kMmaWarp) {
      // ---- tcgen05 issuer: walks the GEMV stages in the consumers' order ----
      if (lane == 0) {
        constexpr uint32_t kIdesc = umma_idesc_bf16(128, FG::UN);
        bool ok = true, fresh = true;
        int pos = 0, buf = 0;
        unsigned uses[2] = {0u, 0u};  // pieces accumulated in each TMEM buffer so far
        SeqIt it;
        seq_begin(P, c, G, it, true);
        while (it.valid) {
          const QmvParams& q = P.ops[it.op].q;
          for (int v = 0; v < it.len; ++v, ++pos) {
            const int s = seq_stage(it, v);
            const StageLoc L = locate(q, s);
            const int st = pos % D;
            if (fresh && uses[buf] > 0 && ok) {
              // The consumers must have read this buffer's previous piece.
              ok = mbar_wait_bounded(&accempty[buf], (uses[buf] - 1) & 1u, nullptr);
              if (!ok) wait_gave_up(P.err, WAIT_CONSUMER_FULL, it.op, s, -2);
            }
            if (ok) {
              ok = mbar_wait_bounded(&full[st], (uint32_t)((pos / D) & 1), nullptr);
              if (!ok) wait_gave_up(P.err, WAIT_CONSUMER_FULL, it.op, s, pos);
            }
            if (ok) {
              tc_fence_after();
              // Weights: 8 K-steps of [16 row groups][2 core matrices] (4 KB
              // each); operand: 8 K-steps of [NT row groups][2 core matrices].
              const uint32_t wa = smem_u32(ring + (size_t)st * FG::STAGE);
              const uint32_t xa = wa + kGemvWarps * FG::PAIRMAX;
              const uint32_t td = s_tmem + (uint32_t)(buf * FG::UN);
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const uint64_t ad = umma_desc_kmajor(wa + kk * 4096, 128, 256);
                const uint64_t bd = umma_desc_kmajor(xa + kk * NT * 256, 128, NT < 2 ? 0 : 256);
                umma_bf16(td, ad, bd, kIdesc, (fresh && kk == 0) ? 0u : 1u);
              }
              umma_commit(&empty[st]);
            } else {
              mbar_arrive(&empty[st]);
            }
            fresh = false;
            if (L.kt == q.seg[L.seg].k_tiles - 1 || s == it.s_end - 1 || v == it.len - 1) {  // end of a piece
              umma_commit(&accfull[buf]);
              ++uses[buf];
              buf ^= 1;
              fresh = true;
            }
          }
          seq_next_chunk(P, c, G, it);
        }
        umma_commit(&issdone);
      }
      return;
    }
  }

  // ---- consumers ----
  pdl_wait();
  float* scr = tail + warp * (kScratch / 4);
  float acc[2][NT][4];
  bool ok = true;
  int pos = 0;
  // tcgen05 path: the TMEM buffer of the next piece and each buffer's use count.
  int cbuf = 0;
  unsigned cuses[2] = {0u, 0u};
  SeqIt it;
  seq_begin(P, c, G, it, false);
  while (it.valid) {
    const int op = it.op;
    if (P.ops[op].kind != OPK_GEMV) break;  // the attention ops, below
    const QmvParams& q = P.ops[op].q;
    const int own = c + it.k * G;
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[rt][nt][i] = 0.f;
    for (int v = 0; v < it.len; ++v, ++pos) {
      const int s = seq_stage(it, v);
      const StageLoc L = locate(q, s);
      const int kts = q.seg[L.seg].k_tiles;
      const int st = pos % D;
      if constexpr (UM) {
        // Stages are the issuer warp's: nothing to do per stage here.
      } else {
        if (ok) {
          ok = mbar_wait_bounded(&full[st], (uint32_t)((pos / D) & 1), nullptr);
          if (!ok) wait_gave_up(P.err, WAIT_CONSUMER_FULL, op, s, pos);
        }
        if (ok) {
          const uint8_t* stage = ring + (size_t)st * FG::STAGE;
          const int fmt = q.seg[L.seg].fmt;
          process_any<SET, NT>(fmt, stage + warp * fmt_pair_bytes(fmt), stage + kGemvWarps * FG::PAIRMAX, scr, lane,
                               acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      if (L.kt == kts - 1 || s == it.s_end - 1 || v == it.len - 1) {  // end of a piece
        if constexpr (UM) {
          // The piece's accumulator: wait for its MMAs, read this warp's 32
          // rows, and hand the buffer back to the issuer.  A piece whose MMAs
          // were skipped (a wait gave up) yields whatever TMEM holds; the
          // error word reports it.
          bool got = mbar_wait_bounded(&accfull[cbuf], cuses[cbuf] & 1u, nullptr);
          if (!got && lane == 0) wait_gave_up(P.err, WAIT_CONSUMER_FULL, op, s, -1);
          ++cuses[cbuf];
          tc_fence_after();
          const uint32_t ta = s_tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cbuf * FG::UN);
#pragma unroll
          for (int c0 = 0; c0 < 8 * NT; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(ta + (uint32_t)c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = c0 + j;
              if (col < 8 * NT) acc[col / (4 * NT)][(col / 4) % NT][col % 4] = __uint_as_float(r[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[cbuf]);
          cbuf ^= 1;
        }
        // What the epilogue reads of earlier ops (norm tables, residual) is
        // ordered before it without a wait here: a group is reduced only
        // after every K stage of it ran, each stage's inputs were acquired
        // by its CTA's producer (flags or count, then the mbarrier hand-off),
        // and the split arrivals release / acquire those CTAs' work.  Every
        // K stage of a group covers every group of the dependency.
        const int i0 = chunk_of(q, L.gstart), i1 = chunk_of(q, L.gstart + kts - 1);
        reduce_and_epilogue<NT, UM>(q, L.grp, own, i0, i1, acc, tail, P.done + op,
                                    P.gflags ? P.gflags + (size_t)op * P.flag_stride : nullptr, epoch);
        consumer_sync();
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[rt][nt][i] = 0.f;
      }
    }
    seq_next_chunk(P, c, G, it);
  }
  if constexpr (UM) {
    // Every consumer warp's TMEM reads are done and every MMA the issuer
    // started has completed (its waits are bounded, so it always gets here):
    // free the columns.
    tc_fence_before();
    consumer_sync();
    if (warp == 0) {
      if (!mbar_wait_bounded(&issdone, 0u, nullptr) && lane == 0)
        wait_gave_up(P.err, WAIT_CONSUMER_FULL, it.valid ? it.op : 255, -3, -3);
      tc_fence_after();
      tmem_dealloc(s_tmem, FG::TCOLS);
    }
  }
  // Attention ops follow every GEMV op of the launch: one chunk = one unit.
  // Every GEMV piece of this CTA is done: the next forward kernel may be
  // scheduled (its CTAs take the slots of CTAs that exit, stream their first
  // weight stages, and wait for this grid's completion before reading
  // anything it writes), so its launch overlaps the attention tail.
  if (it.valid && Pg.trigger_after_gemv) pdl_launch_dependents();
  static_assert(FG::RING % 16 == 0 && FG::RING > kAttnParamBytes, "ring too small for attention units");
  while (it.valid) {
    if (s_ops[it.op].kind == OPK_GEMV) {  // schedules put attention last: a GEMV op here is a bad schedule
      if (threadIdx.x == 0) atomicOr(Pg.err, DEV_ERR_BAD_ARGUMENT);
      break;
    }
    for (int u = it.s0; u < it.s_end; ++u)
      attn_op_unit<NT>(s_ops, Pg.done, Pg.gflags, Pg.flag_stride, Pg.err, it.op, u, ring, FG::RING, epoch);
    seq_next_chunk(P, c, G, it);
  }
}

// ---------------------------------------------------------------------------
// Repack: GGUF blocks -> pair tiles.  One warp per 16-row tile x KT columns.
// ---------------------------------------------------------------------------
SPEC_DEV int code_at(const uint8_t* row, int fmt, int k) {
  if (fmt == WF_Q4_K || fmt == WF_Q5_K) {
    const int bb = fmt == WF_Q4_K ? 144 : 176, qoff = fmt == WF_Q4_K ? 16 : 48;
    const uint8_t* b = row + (k >> 8) * bb;
    const int kk = k & 255, c = kk >> 6, l = kk & 31, hi = (kk & 63) >> 5;
    const uint8_t byte = b[qoff + 32 * c + l];
    return hi ? (byte >> 4) : (byte & 15);
  }
  if (fmt == WF_Q6_K) {
    const uint8_t* b = row + (k >> 8) * 210;
    const int kk = k & 255, n = kk >> 7, r = kk & 127, j = r >> 5, l = r & 31;
    const uint8_t lb = b[64 * n + l + (j & 1) * 32];
    return (j < 2) ? (lb & 15) : (lb >> 4);
  }
  if (fmt == WF_Q8_0) {
    const uint8_t* b = row + (k >> 5) * 34;
    return b[2 + (k & 31)];
  }
  return 0;
}
SPEC_DEV int high_at(const uint8_t* row, int fmt, int k) {
  if (fmt == WF_Q5_K) {
    const uint8_t* b = row + (k >> 8) * 176;
    const int kk = k & 255, c = kk >> 6, l = kk & 31, hi = (kk & 63) >> 5;
    return (b[16 + l] >> (2 * c + hi)) & 1;
  }
  if (fmt == WF_Q6_K) {
    const uint8_t* b = row + (k >> 8) * 210;
    const int kk = k & 255, n = kk >> 7, r = kk & 127, j = r >> 5, l = r & 31;
    return (b[128 + 32 * n + l] >> (2 * j)) & 3;
  }
  return 0;
}

// Row/column of nibble position p (0..7) of lane (g,t)'s word for one k-step.
SPEC_DEV void nib_pos(int p, int g, int t, int& row, int& col) {
  const int rsel = p & 1;          // n0,n2 -> row g ; n1,n3 -> row g+8 (for p < 4)
  const int csel = (p >> 1) & 1;   // n0,n1 -> col 2t ; n2,n3 -> col 2t+8
  const int hi = p >> 2;           // n4..n7: +1 column
  row = g + (rsel ? 8 : 0);
  col = 2 * t + (csel ? 8 : 0) + hi;
}

__global__ void repack_kernel(const uint8_t* raw, int fmt, int N, int K, uint8_t* tiles) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rt16 = blockIdx.x;  // 16-row tile index
  const int kt = blockIdx.y;
  const int KT = fmt_kt(fmt), TB = fmt_tile_bytes(fmt);
  const int be = fmt_block_elems(fmt), bb = fmt_block_bytes(fmt);
  const size_t row_bytes = (size_t)(K / be) * bb;
  const int k_tiles = K / KT;
  // Layout [group][k-tile][warp][16-row tile]: the 4 pair tiles of one
  // stage (128 rows x one k-tile) are contiguous, so a stage is one bulk copy.
  const int pair = rt16 >> 1;
  uint8_t* out = tiles + (((((size_t)(pair >> 2) * k_tiles + kt) * kGemvWarps + (pair & 3)) * 2) + (rt16 & 1)) * TB;
  const int r0 = rt16 * 16;
  const int kbase = kt * KT;
  if (fmt == WF_BF16) {
    // A stage (128 rows x 128 columns, 32 KB) in the tensor core's K-major
    // no-swizzle canonical layout: [K-step of 16][8-row group][8-column
    // half][8 rows x 16 bytes].  This warp writes its 16 rows, 16 bytes
    // (8 columns of one row) per lane and step.
    uint8_t* stage = tiles + ((size_t)(rt16 >> 3) * k_tiles + kt) * (kGemvWarps * 2 * TB);
    const int rbase = (rt16 & 7) * 16;
    for (int i = lane; i < 16 * (KT / 8); i += 32) {
      const int row = i / (KT / 8), c8 = i % (KT / 8);
      const int rr = rbase + row, k0 = c8 * 8;
      const uint8_t* src = raw + (size_t)(r0 + row) * row_bytes + (size_t)(kbase + k0) * 2;
      uint4 v;
      uint8_t* vb = reinterpret_cast<uint8_t*>(&v);
      for (int b = 0; b < 16; ++b) vb[b] = src[b];
      *reinterpret_cast<uint4*>(stage + ((k0 >> 4) * 16 + (rr >> 3)) * 256 + ((k0 >> 3) & 1) * 128 + (rr & 7) * 16) = v;
    }
    return;
  }
  if (fmt == WF_Q8_0) {
    for (int s = 0; s < KT / 16; ++s) {
      uint32_t w[2];
      for (int h = 0; h < 2; ++h) {
        uint32_t acc = 0;
        for (int byte = 0; byte < 4; ++byte) {
          const int row = g + ((byte >> 1) ? 8 : 0), col = 2 * t + (h ? 8 : 0) + (byte & 1);
          const uint8_t* rowp = raw + (size_t)(r0 + row) * row_bytes;
          acc |= (uint32_t)code_at(rowp, fmt, kbase + 16 * s + col) << (8 * byte);
        }
        w[h] = acc;
      }
      uint32_t* dst = reinterpret_cast<uint32_t*>(out + (s >> 1) * 512 + lane * 16 + (s & 1) * 8);
      dst[0] = w[0];
      dst[1] = w[1];
    }
    if (lane < 16) {
      const uint8_t* rowp = raw + (size_t)(r0 + lane) * row_bytes;
      for (int b = 0; b < 4; ++b) {
        const uint8_t* blk = rowp + (size_t)((kbase >> 5) + b) * 34;
        out[2048 + (lane * 4 + b) * 2] = blk[0];
        out[2048 + (lane * 4 + b) * 2 + 1] = blk[1];
      }
    }
    return;
  }
  // K-quants: low nibbles in A-fragment order.
  for (int s = 0; s < 16; ++s) {
    uint32_t w = 0;
    for (int p = 0; p < 8; ++p) {
      int row, col;
      nib_pos(p, g, t, row, col);
      const uint8_t* rowp = raw + (size_t)(r0 + row) * row_bytes;
      const int k = kbase + 16 * s + col;
      w |= (uint32_t)code_at(rowp, fmt, k) << (4 * p);
    }
    *reinterpret_cast<uint32_t*>(out + (s >> 2) * 512 + lane * 16 + (s & 3) * 4) = w;
  }
  if (fmt == WF_Q5_K) {
    for (int j = 0; j < 4; ++j) {
      uint32_t hw = 0;
      for (int i = 0; i < 4; ++i) {
        const int s = 4 * j + i;
        for (int p = 0; p < 8; ++p) {
          int row, col;
          nib_pos(p, g, t, row, col);
          const uint8_t* rowp = raw + (size_t)(r0 + row) * row_bytes;
          const int bit = high_at(rowp, fmt, kbase + 16 * s + col);
          const int pos = (p < 4) ? (4 * i + p) : (16 + 4 * i + (p - 4));
          hw |= (uint32_t)bit << pos;
        }
      }
      *reinterpret_cast<uint32_t*>(out + 2048 + j * 128 + lane * 4) = hw;
    }
  }
  if (fmt == WF_Q6_K) {
    for (int pr = 0; pr < 8; ++pr) {
      uint32_t hw = 0;
      for (int i = 0; i < 2; ++i) {
        const int s = 2 * pr + i;
        for (int p = 0; p < 8; ++p) {
          int row, col;
          nib_pos(p, g, t, row, col);
          const uint8_t* rowp = raw + (size_t)(r0 + row) * row_bytes;
          const int v = high_at(rowp, fmt, kbase + 16 * s + col);
          const int pos = (p < 4) ? 2 * (4 * i + p) : 16 + 2 * (4 * i + (p - 4));
          hw |= (uint32_t)v << pos;
        }
      }
      *reinterpret_cast<uint32_t*>(out + 2048 + pr * 128 + lane * 4) = hw;
    }
  }
  if (lane < 16) {
    const uint8_t* blk = raw + (size_t)(r0 + lane) * row_bytes + (size_t)(kbase >> 8) * bb;
    if (fmt == WF_Q4_K || fmt == WF_Q5_K) {
      const int off = fmt == WF_Q4_K ? 2048 : 2560;
      for (int i = 0; i < 16; ++i) out[off + lane * 16 + i] = blk[i];
    } else {  // Q6_K
      for (int i = 0; i < 16; ++i) out[3072 + lane * 16 + i] = blk[192 + i];
      out[3328 + lane * 2] = blk[208];
      out[3328 + lane * 2 + 1] = blk[209];
    }
  }
}

template <int SET, int NT>
struct FwdInst {
  struct Occ {
    int bps[16] = {0};
    int sms[16] = {0};
  };
  static Occ& occ() {
    static Occ o;
    return o;
  }
  static cudaError_t prepare(int dev) {
    int* bps = occ().bps;
    int* sms = occ().sms;
    if (bps[dev]) return cudaSuccess;
    constexpr int smem = FGeo<SET, NT>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(fwd_kernel<SET, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int b = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fwd_kernel<SET, NT>, FGeo<SET, NT>::THREADS, smem);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms[dev] = n;
    bps[dev] = b > 0 ? b : 1;
    return cudaSuccess;
  }
  static cudaError_t launch(const FwdParams& p, cudaStream_t stream, bool pdl) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16) return cudaErrorInvalidDevice;
    cudaError_t e = prepare(dev);
    if (e != cudaSuccess) return e;
    const int* bps = occ().bps;
    const int* sms = occ().sms;
    int grid = bps[dev] * sms[dev];
    if (const char* env = getenv("SPEC_B200_GEMV_CTAS_PER_SM")) {
      const int v = atoi(env);
      if (v > 0 && v < bps[dev]) grid = v * sms[dev];
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(FGeo<SET, NT>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = FGeo<SET, NT>::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.cooperative) {  // every CTA resident at once, or the launch fails
      attr[1].id = cudaLaunchAttributeCooperative;
      attr[1].val.cooperative = 1;
      cfg.numAttrs = 2;
    }
    return cudaLaunchKernelEx(&cfg, fwd_kernel<SET, NT>, p);
  }
};

template <int SET>
cudaError_t launch_set(const FwdParams& p, int M, cudaStream_t s, bool pdl) {
  const int nt = nt_for_rows(M);
  if (nt == 1) return FwdInst<SET, 1>::launch(p, s, pdl);
  if (nt == 2) return FwdInst<SET, 2>::launch(p, s, pdl);
  if (nt == 4) return FwdInst<SET, 4>::launch(p, s, pdl);
  return FwdInst<SET, 8>::launch(p, s, pdl);
}

// Instantiated format sets: GGUF K-quant mixes (with the Q8_0 fallback for
// K % 256 != 0) and BF16.
constexpr int kSetK4 = FS_Q4K | FS_Q6K | FS_Q80;
constexpr int kSetK5 = FS_Q5K | FS_Q6K | FS_Q80;
constexpr int kSetBF = FS_BF16;

}  // namespace

int fwd_attn_keys_per_pass(int set, int M, int hd, int chunk) {
  const int nt = nt_for_rows(M);
  int ring = 0;
  auto pick = [&](auto tag) {
    constexpr int S = decltype(tag)::value;
    ring = nt == 1 ? FGeo<S, 1>::RING : nt == 2 ? FGeo<S, 2>::RING : nt == 4 ? FGeo<S, 4>::RING : FGeo<S, 8>::RING;
  };
  if (set == kSetK4) pick(std::integral_constant<int, kSetK4>{});
  else if (set == kSetK5) pick(std::integral_constant<int, kSetK5>{});
  else if (set == kSetBF) pick(std::integral_constant<int, kSetBF>{});
  else return 0;
  return attn_keys_per_pass(ring - kAttnParamBytes, hd, chunk);
}

int fwd_fmt_set_for(int bits) {
  if ((bits & ~kSetK4) == 0) return kSetK4;
  if ((bits & ~kSetK5) == 0) return kSetK5;
  if ((bits & ~kSetBF) == 0) return kSetBF;
  return 0;
}

int fwd_ctas_per_sm(int set) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaErrorInvalidValue;
  if (set == kSetK4) {
    e = FwdInst<kSetK4, 1>::prepare(dev);
    if (e == cudaSuccess) return FwdInst<kSetK4, 1>::occ().bps[dev];
  } else if (set == kSetK5) {
    e = FwdInst<kSetK5, 1>::prepare(dev);
    if (e == cudaSuccess) return FwdInst<kSetK5, 1>::occ().bps[dev];
  } else if (set == kSetBF) {
    e = FwdInst<kSetBF, 1>::prepare(dev);
    if (e == cudaSuccess) return FwdInst<kSetBF, 1>::occ().bps[dev];
  }
  return 3;
}

cudaError_t launch_fwd(const FwdParams& p, int fmt_set, int M, cudaStream_t s, bool pdl) {
  if (M < 1 || M > kMaxRows || p.n_ops < 1 || p.n_ops > kMaxLaunchOps) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.ops) % 16) return cudaErrorMisalignedAddress;
  if (fmt_set == kSetK4) return launch_set<kSetK4>(p, M, s, pdl);
  if (fmt_set == kSetK5) return launch_set<kSetK5>(p, M, s, pdl);
  if (fmt_set == kSetBF) return launch_set<kSetBF>(p, M, s, pdl);
  return cudaErrorNotSupported;
}

namespace {
// One thread: waits until this rank's logits arrival counter reaches the
// forward's target (every rank's LM-head groups stored), bounded by the
// usual 2 s; on timeout it records WAIT_TP_PEERS and returns.
__global__ void tp_logits_wait_kernel(const unsigned long long* counter, const unsigned long long* target,
                                      unsigned* err) {
  if (threadIdx.x != 0) return;
  const unsigned long long want = *target;
  const unsigned long long t0 = global_timer_ns();
  for (unsigned i = 0;; ++i) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
    if (v >= want) return;
    if ((i & 255u) == 255u && global_timer_ns() - t0 > kMbarTimeoutNs) {
      wait_gave_up(err, WAIT_TP_PEERS, 255, 0, (int)(v & 0x7fffffff));
      return;
    }
  }
}
}  // namespace

cudaError_t launch_tp_logits_wait(const unsigned long long* counter, const unsigned long long* target, unsigned* err,
                                  cudaStream_t s) {
  tp_logits_wait_kernel<<<1, 32, 0, s>>>(counter, target, err);
  return cudaGetLastError();
}

cudaError_t launch_repack(const uint8_t* raw, int fmt, int N, int K, uint8_t* tiles, cudaStream_t s) {
  const int KT = fmt_kt(fmt);
  if (N % 32 || K % KT || fmt_tile_bytes(fmt) == 0) return cudaErrorInvalidValue;
  repack_kernel<<<dim3(N / 16, K / KT), 32, 0, s>>>(raw, fmt, N, K, tiles);
  return cudaGetLastError();
}

}  // namespace specb200
