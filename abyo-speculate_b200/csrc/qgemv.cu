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
//    a 32-row slice and streams its pair tiles with TMA bulk copies
//    (cp.async.bulk -> shared, mbarrier completion) through a 2-3 stage ring.
//  * Codes become f16 with one LOP3 each (magic 0x6400: value = 1024 + q),
//    feed mma.sync with the activation fragments, and the accumulator is
//    seeded with -offset * (sum of the activations of that sub-block), so the
//    tensor core returns exactly sum(q * x) for the sub-block.  The sub-block
//    scale (and K-quant min term) is applied in f32 afterwards:
//        acc += s_row * D - c_row * xsum.
//    Products q*x are exact in the tensor core (q <= 63, x f16), so the only
//    roundings are the f16 activations and f32 accumulation.
//  * K is split into S fixed chunks; partial sums go to scratch and the last
//    CTA of a 128-row group adds them in split order 0..S-1, then runs the
//    fused epilogue.  Nothing depends on M except which fragment columns are
//    live, so row r's result is bit-identical for any M (batched == sequential).
//  * Programmatic dependent launch: a CTA issues its first weight copies, then
//    waits for the previous kernel (griddepcontrol.wait) before touching
//    activations, so weight streaming overlaps the predecessor's tail.
#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {

namespace {

SPEC_DEV float h2f_bits(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu))); }

// ---------------------------------------------------------------------------
// Activation operand access
// ---------------------------------------------------------------------------
template <int NT>
SPEC_DEV void load_b(const QmvParams& p, int ks, int lane, uint32_t (&b)[NT][2]) {
  const int g = lane >> 2;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    if (nt * 8 + g < p.M) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p.xfrag) + ((size_t)ks * NT + nt) * 32 + lane);
      b[nt][0] = v.x;
      b[nt][1] = v.y;
    } else {
      b[nt][0] = 0u;
      b[nt][1] = 0u;
    }
  }
}

template <int NT>
SPEC_DEV float2 load_xs(const float* xs, int blk, int nt, int lane) {
  const int t = lane & 3;
  return __ldg(reinterpret_cast<const float2*>(xs + (size_t)blk * (8 * NT) + nt * 8 + 2 * t));
}

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
// eight 4-bit codes: value = 1024 + code.
SPEC_DEV void a_from_nibbles(uint32_t w, uint32_t (&a)[4]) {
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  a[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x64006400u);
  a[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x64006400u);
  a[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x64006400u);
}

template <int NT>
SPEC_DEV void mma_sub(const uint32_t (&a)[4], const uint32_t (&b)[NT][2], int nt, float c0, float c1, float (&d)[4]) {
  mma_f16(d, a[0], a[1], a[2], a[3], b[nt][0], b[nt][1], c0, c1, c0, c1);
}
template <int NT>
SPEC_DEV void mma_acc(const uint32_t (&a)[4], const uint32_t (&b)[NT][2], int nt, float (&d)[4]) {
  mma_f16(d, a[0], a[1], a[2], a[3], b[nt][0], b[nt][1], d[0], d[1], d[2], d[3]);
}

// ---------------------------------------------------------------------------
// Per-format pair-tile processing.  `tp` = pair tile in shared memory,
// `ks0` = global k-step (16 columns) of the tile's first column.
// ---------------------------------------------------------------------------
template <int NT>
SPEC_DEV void tile_q4k(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 2304;
  const int g = lane >> 2;
  uint4 meta[2][2];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt) {
    meta[rt][0] = *reinterpret_cast<const uint4*>(tp + rt * TB + 2048 + g * 16);
    meta[rt][1] = *reinterpret_cast<const uint4*>(tp + rt * TB + 2048 + (g + 8) * 16);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t bq[4][NT][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) load_b<NT>(p, ks0 + 4 * j + i, lane, bq[i]);
    float2 xs[2][NT];
#pragma unroll
    for (int sb = 0; sb < 2; ++sb)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xs[sb][nt] = load_xs<NT>(p.xsum32, ks0 / 2 + 2 * j + sb, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const uint32_t wv[4] = {qw.x, qw.y, qw.z, qw.w};
#pragma unroll
      for (int sb = 0; sb < 2; ++sb) {
        const int b = 2 * j + sb;
        float s[2], c[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          int sc, mn;
          k4_scale_min(meta[rt][r], b, sc, mn);
          s[r] = h2f_bits(meta[rt][r].x) * (float)sc;
          c[r] = h2f_bits(meta[rt][r].x >> 16) * (float)mn;
        }
        uint32_t a0[4], a1[4];
        a_from_nibbles(wv[2 * sb], a0);
        a_from_nibbles(wv[2 * sb + 1], a1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float c0 = -1024.f * xs[sb][nt].x, c1 = -1024.f * xs[sb][nt].y;
          float d[4];
          mma_sub<NT>(a0, bq[2 * sb], nt, c0, c1, d);
          mma_acc<NT>(a1, bq[2 * sb + 1], nt, d);
          float* ac = acc[rt][nt];
          ac[0] = fmaf(s[0], d[0], fmaf(-c[0], xs[sb][nt].x, ac[0]));
          ac[1] = fmaf(s[0], d[1], fmaf(-c[0], xs[sb][nt].y, ac[1]));
          ac[2] = fmaf(s[1], d[2], fmaf(-c[1], xs[sb][nt].x, ac[2]));
          ac[3] = fmaf(s[1], d[3], fmaf(-c[1], xs[sb][nt].y, ac[3]));
        }
      }
    }
  }
}

template <int NT>
SPEC_DEV void tile_q5k(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 2816;
  const int g = lane >> 2;
  uint4 meta[2][2];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt) {
    meta[rt][0] = *reinterpret_cast<const uint4*>(tp + rt * TB + 2560 + g * 16);
    meta[rt][1] = *reinterpret_cast<const uint4*>(tp + rt * TB + 2560 + (g + 8) * 16);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t bq[4][NT][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) load_b<NT>(p, ks0 + 4 * j + i, lane, bq[i]);
    float2 xs[2][NT];
#pragma unroll
    for (int sb = 0; sb < 2; ++sb)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xs[sb][nt] = load_xs<NT>(p.xsum32, ks0 / 2 + 2 * j + sb, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const uint32_t hw = *reinterpret_cast<const uint32_t*>(tp + rt * TB + 2048 + j * 128 + lane * 4);
      const uint32_t wv[4] = {qw.x, qw.y, qw.z, qw.w};
#pragma unroll
      for (int sb = 0; sb < 2; ++sb) {
        const int b = 2 * j + sb;
        float s[2], c[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          int sc, mn;
          k4_scale_min(meta[rt][r], b, sc, mn);
          s[r] = h2f_bits(meta[rt][r].x) * (float)sc;
          c[r] = h2f_bits(meta[rt][r].x >> 16) * (float)mn;
        }
        uint32_t a[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * sb + h;  // k-step within the group of 4
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t base = lop3_and_or(wv[i] >> (4 * jj), 0x000F000Fu, 0x64006400u);
            a[h][jj] = lop3_or_and(base, shift_signed(hw, 4 * i + jj - 4), 0x00100010u);
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float c0 = -1024.f * xs[sb][nt].x, c1 = -1024.f * xs[sb][nt].y;
          float d[4];
          mma_sub<NT>(a[0], bq[2 * sb], nt, c0, c1, d);
          mma_acc<NT>(a[1], bq[2 * sb + 1], nt, d);
          float* ac = acc[rt][nt];
          ac[0] = fmaf(s[0], d[0], fmaf(-c[0], xs[sb][nt].x, ac[0]));
          ac[1] = fmaf(s[0], d[1], fmaf(-c[0], xs[sb][nt].y, ac[1]));
          ac[2] = fmaf(s[1], d[2], fmaf(-c[1], xs[sb][nt].x, ac[2]));
          ac[3] = fmaf(s[1], d[3], fmaf(-c[1], xs[sb][nt].y, ac[3]));
        }
      }
    }
  }
}

template <int NT>
SPEC_DEV void tile_q6k(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 3360;
  const int g = lane >> 2;
  uint4 scl[2][2];
  float dd[2][2];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt) {
    scl[rt][0] = *reinterpret_cast<const uint4*>(tp + rt * TB + 3072 + g * 16);
    scl[rt][1] = *reinterpret_cast<const uint4*>(tp + rt * TB + 3072 + (g + 8) * 16);
    dd[rt][0] = h2f_bits(*reinterpret_cast<const uint16_t*>(tp + rt * TB + 3328 + g * 2));
    dd[rt][1] = h2f_bits(*reinterpret_cast<const uint16_t*>(tp + rt * TB + 3328 + (g + 8) * 2));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t bq[4][NT][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) load_b<NT>(p, ks0 + 4 * j + i, lane, bq[i]);
    float2 xs[4][NT];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xs[i][nt] = load_xs<NT>(p.xsum16, ks0 + 4 * j + i, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const uint32_t wv[4] = {qw.x, qw.y, qw.z, qw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ksl = 4 * j + i;  // k-step within the superblock = sub-block index
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(tp + rt * TB + 2048 + (ksl >> 1) * 128 + lane * 4);
        const int ip = ksl & 1;
        uint32_t a[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t base = lop3_and_or(wv[i] >> (4 * jj), 0x000F000Fu, 0x64006400u);
          a[jj] = lop3_or_and(base, shift_signed(hw, 2 * (4 * ip + jj) - 4), 0x00300030u);
        }
        const uint32_t sw0 = (ksl < 4 ? scl[rt][0].x : ksl < 8 ? scl[rt][0].y : ksl < 12 ? scl[rt][0].z : scl[rt][0].w);
        const uint32_t sw1 = (ksl < 4 ? scl[rt][1].x : ksl < 8 ? scl[rt][1].y : ksl < 12 ? scl[rt][1].z : scl[rt][1].w);
        const float s0 = dd[rt][0] * (float)(int8_t)((sw0 >> (8 * (ksl & 3))) & 0xff);
        const float s1 = dd[rt][1] * (float)(int8_t)((sw1 >> (8 * (ksl & 3))) & 0xff);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float d[4];
          mma_sub<NT>(a, bq[i], nt, -1056.f * xs[i][nt].x, -1056.f * xs[i][nt].y, d);
          float* ac = acc[rt][nt];
          ac[0] = fmaf(s0, d[0], ac[0]);
          ac[1] = fmaf(s0, d[1], ac[1]);
          ac[2] = fmaf(s1, d[2], ac[2]);
          ac[3] = fmaf(s1, d[3], ac[3]);
        }
      }
    }
  }
}

template <int NT>
SPEC_DEV void tile_q80(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 2176;
  const int g = lane >> 2;
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // one Q8_0 block (32 columns) per j
    uint32_t bq[2][NT][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) load_b<NT>(p, ks0 + 2 * j + i, lane, bq[i]);
    float2 xs[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xs[nt] = load_xs<NT>(p.xsum32, ks0 / 2 + j, nt, lane);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 qw = *reinterpret_cast<const uint4*>(tp + rt * TB + j * 512 + lane * 16);
      const float s0 = h2f_bits(*reinterpret_cast<const uint16_t*>(tp + rt * TB + 2048 + (g * 4 + j) * 2));
      const float s1 = h2f_bits(*reinterpret_cast<const uint16_t*>(tp + rt * TB + 2048 + ((g + 8) * 4 + j) * 2));
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
        mma_sub<NT>(a[0], bq[0], nt, -1152.f * xs[nt].x, -1152.f * xs[nt].y, d);
        mma_acc<NT>(a[1], bq[1], nt, d);
        float* ac = acc[rt][nt];
        ac[0] = fmaf(s0, d[0], ac[0]);
        ac[1] = fmaf(s0, d[1], ac[1]);
        ac[2] = fmaf(s1, d[2], ac[2]);
        ac[3] = fmaf(s1, d[3], ac[3]);
      }
    }
  }
}

template <int NT>
SPEC_DEV void tile_bf16(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  constexpr int TB = 4096;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    uint32_t bq[NT][2];
    load_b<NT>(p, ks0 + s, lane, bq);
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint4 a = *reinterpret_cast<const uint4*>(tp + rt * TB + s * 512 + lane * 16);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* ac = acc[rt][nt];
        float d[4] = {ac[0], ac[1], ac[2], ac[3]};
        mma_bf16(d, a.x, a.y, a.z, a.w, bq[nt][0], bq[nt][1], d[0], d[1], d[2], d[3]);
        ac[0] = d[0];
        ac[1] = d[1];
        ac[2] = d[2];
        ac[3] = d[3];
      }
    }
  }
}

template <int F, int NT>
SPEC_DEV void process_tile(const uint8_t* tp, int ks0, const QmvParams& p, int lane, float (&acc)[2][NT][4]) {
  if constexpr (F == WF_Q4_K) tile_q4k<NT>(tp, ks0, p, lane, acc);
  else if constexpr (F == WF_Q5_K) tile_q5k<NT>(tp, ks0, p, lane, acc);
  else if constexpr (F == WF_Q6_K) tile_q6k<NT>(tp, ks0, p, lane, acc);
  else if constexpr (F == WF_Q8_0) tile_q80<NT>(tp, ks0, p, lane, acc);
  else tile_bf16<NT>(tp, ks0, p, lane, acc);
}

// ---------------------------------------------------------------------------
// Per-warp streaming loop over this warp's pair tiles.
// ---------------------------------------------------------------------------
template <int F, int NT>
SPEC_DEV void gemv_segment(const QmvParams& p, const WSeg& sg, int group_in_seg, int split, uint8_t* smem,
                           uint64_t* bars, float (&acc)[2][NT][4]) {
  constexpr int PAIR = fmt_pair_bytes(F);
  constexpr int ST = fmt_stages(F);
  constexpr int KSTEPS = fmt_kt(F) / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rowpair = group_in_seg * kGemvWarps + warp;
  const int kt0 = split * sg.tiles_per_split;
  const int cnt = sg.tiles_per_split;
  const uint8_t* src = sg.w + ((size_t)rowpair * sg.k_tiles + kt0) * PAIR;
  uint8_t* ring = smem + (size_t)warp * ST * PAIR;
  uint64_t* bar = bars + warp * 4;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < ST; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0) {
    const int n0 = cnt < ST ? cnt : ST;
    for (int i = 0; i < n0; ++i) {
      mbar_arrive_expect_tx(&bar[i], PAIR);
      tma_bulk_g2s(ring + i * PAIR, src + (size_t)i * PAIR, PAIR, &bar[i]);
    }
  }
  // Everything above touches only weights; activations come from the
  // previous kernel.
  pdl_wait();

#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[rt][nt][i] = 0.f;

  int done = 0;
  bool ok = true;
  for (int i = 0; i < cnt; ++i) {
    const int slot = i % ST;
    const uint32_t par = (uint32_t)((i / ST) & 1);
    if (!mbar_wait_bounded(&bar[slot], par, p.err)) {
      ok = false;
      break;
    }
    process_tile<F, NT>(ring + slot * PAIR, (kt0 + i) * KSTEPS, p, lane, acc);
    __syncwarp();
    if (lane == 0 && i + ST < cnt) {
      mbar_arrive_expect_tx(&bar[slot], PAIR);
      tma_bulk_g2s(ring + slot * PAIR, src + (size_t)(i + ST) * PAIR, PAIR, &bar[slot]);
    }
    done = i + 1;
  }
  if (!ok) {
    // Drain whatever copies are still in flight (bounded) before the CTA
    // may exit and release its shared memory.
    const int issued = (cnt < done + ST) ? cnt : done + ST;
    for (int i = done; i < issued; ++i) mbar_wait_bounded(&bar[i % ST], (uint32_t)((i / ST) & 1), nullptr);
  }
}

// ---------------------------------------------------------------------------
// Operand-fragment writer used by the producing epilogues.
// ---------------------------------------------------------------------------
SPEC_DEV void frag_store(uint32_t* frag, int nt_total, int m, int k, uint16_t bits) {
  const int s = k >> 4, kk = k & 15, nt = m >> 3, g = m & 7;
  const int t = (kk & 7) >> 1, slot = kk >> 3, lo = kk & 1;
  const size_t hidx = ((size_t)((s * nt_total + nt) * 32 + g * 4 + t)) * 4 + slot * 2 + lo;
  reinterpret_cast<uint16_t*>(frag)[hidx] = bits;
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

// Writes value v for (row m, column k) of the next operand and accumulates
// the per-16 / per-32 column sums.  Called by a full warp whose lanes hold 32
// consecutive columns starting at a multiple of 32 (k = k0 + lane).
SPEC_DEV void emit_operand_warp(uint32_t* frag, float* xs16, float* xs32, int nt_total, int m, int k, float v,
                                int bf16, int lane) {
  float back;
  const uint16_t bits = round_act(v, bf16, back);
  frag_store(frag, nt_total, m, k, bits);
  float s16 = back;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
  const int w16 = 8 * nt_total;
  if ((lane & 15) == 0) xs16[(size_t)(k >> 4) * w16 + m] = s16;
  if (lane == 0) xs32[(size_t)(k >> 5) * w16 + m] = s32;
}

// ---------------------------------------------------------------------------
// Split-K reduction and fused epilogues.
// ---------------------------------------------------------------------------
template <int NT>
SPEC_DEV void reduce_and_epilogue(const QmvParams& p, int group, int split, float (&acc)[2][NT][4], float* ys) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  __shared__ int s_last;
  __shared__ float s_rinv[kMaxRows];
  __shared__ float s_red[kGemvWarps][kMaxRows];
  const int M = p.M;

  if (p.S > 1) {
    const size_t per = (size_t)kGroupRows * 8 * NT;
    float* mine = p.part + ((size_t)split * gridDim.x + group) * per;
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        __stcg(reinterpret_cast<float4*>(mine + ((size_t)((warp * 2 + rt) * NT + nt) * 32 + lane) * 4),
               make_float4(acc[rt][nt][0], acc[rt][nt][1], acc[rt][nt][2], acc[rt][nt][3]));
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(&p.counters[group], 1);
      s_last = (prev == p.S - 1);
      if (s_last) p.counters[group] = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[rt][nt][i] = 0.f;
    for (int s = 0; s < p.S; ++s) {
      const float* ps = p.part + ((size_t)s * gridDim.x + group) * per;
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(ps + ((size_t)((warp * 2 + rt) * NT + nt) * 32 + lane) * 4));
          acc[rt][nt][0] += v.x;
          acc[rt][nt][1] += v.y;
          acc[rt][nt][2] += v.z;
          acc[rt][nt][3] += v.w;
        }
    }
  }
  __syncthreads();  // every warp is done with its TMA ring: reuse as ys
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = warp * 32 + rt * 16 + g + ((i >> 1) ? 8 : 0);
        const int col = nt * 8 + 2 * t + (i & 1);
        if (col < M) ys[col * kGroupRows + row] = acc[rt][nt][i];
      }
  if (tid < M) {
    float r = 1.f;
    if (p.ss_in) {
      float ms = 0.f;
      for (int q = 0; q < p.ss_groups; ++q) ms += p.ss_in[q * kSsStride + tid];
      r = 1.f / sqrtf(ms * p.ss_inv_dim + p.eps);
    }
    s_rinv[tid] = r;
  }
  __syncthreads();

  const int n0 = group * kGroupRows;
  if (p.epi == EPI_STORE) {
    for (int idx = tid; idx < M * kGroupRows; idx += blockDim.x) {
      const int m = idx / kGroupRows, j = idx % kGroupRows, n = n0 + j;
      float v = ys[m * kGroupRows + j] * s_rinv[m];
      if (p.bias) v += p.bias[n];
      p.out[(size_t)m * p.ld_out + n] = v;
    }
  } else if (p.epi == EPI_QKV) {
    const int hd = p.head_dim, nq = p.n_q_heads, nkv = p.n_kv_heads;
    const int G = nq / nkv, R = M * G, half = hd / 2;
    for (int idx = tid; idx < M * kGroupRows; idx += blockDim.x) {
      const int m = idx / kGroupRows, j = idx % kGroupRows, n = n0 + j;
      const int d = n % hd, head = n / hd;
      float x = ys[m * kGroupRows + j] * s_rinv[m];
      if (p.bias) x += p.bias[n];
      const bool is_v = head >= nq + nkv;
      float out = x;
      if (!is_v) {
        int jp, ci;
        if (p.rope_interleaved) {
          jp = j ^ 1;
          ci = d >> 1;
        } else {
          jp = d < half ? j + half : j - half;
          ci = d < half ? d : d - half;
        }
        float y = ys[m * kGroupRows + jp] * s_rinv[m];
        if (p.bias) y += p.bias[n0 + jp];
        const int pos = p.positions[m];
        const float cs = p.rope_cos[(size_t)pos * half + ci], sn = p.rope_sin[(size_t)pos * half + ci];
        const bool first = p.rope_interleaved ? ((d & 1) == 0) : (d < half);
        out = first ? (x * cs - y * sn) : (y * sn + x * cs);
      }
      float back;
      const uint16_t bits = round_act(out, p.act_bf16, back);
      if (head < nq) {
        const int kvh = head / G, gq = head % G, r = m * G + gq;
        reinterpret_cast<uint16_t*>(p.qbuf)[((size_t)kvh * R + r) * hd + d] = bits;
      } else if (!is_v) {
        const int kvh = head - nq;
        reinterpret_cast<uint16_t*>(p.kcache)[((size_t)kvh * p.t_max + p.kv_slots[m]) * hd + d] = bits;
      } else {
        const int kvh = head - nq - nkv;
        reinterpret_cast<uint16_t*>(p.vcache)[((size_t)kvh * p.t_max + p.kv_slots[m]) * hd + d] = bits;
      }
    }
  } else if (p.epi == EPI_RESID) {
    const int H = p.n_rows;
    const int n = n0 + tid;  // 128 threads, one column each
    for (int m = 0; m < M; ++m) {
      const float hv = p.h[(size_t)m * H + n] + ys[m * kGroupRows + tid];
      p.h[(size_t)m * H + n] = hv;
      const float sq = warp_sum(hv * hv);
      if (lane == 0) s_red[warp][m] = sq;
      if (p.next_frag) {
        const float v = p.next_norm ? hv * p.next_norm[n] : hv;
        emit_operand_warp(p.next_frag, p.next_xsum16, p.next_xsum32, NT, m, n, v, p.act_bf16, lane);
      }
    }
    __syncthreads();
    if (tid < M) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) ss += s_red[w][tid];
      p.ss_out[group * kSsStride + tid] = ss;
    }
  } else if (p.epi == EPI_SILU) {
    if (tid < 64) {
      const int f = group * 64 + tid;
      for (int m = 0; m < M; ++m) {
        const float gv = ys[m * kGroupRows + tid] * s_rinv[m];
        const float uv = ys[m * kGroupRows + tid + 64] * s_rinv[m];
        const float a = gv / (1.f + expf(-gv)) * uv;
        emit_operand_warp(p.next_frag, p.next_xsum16, p.next_xsum32, NT, m, f, a, p.act_bf16, lane);
      }
    }
  }
}

template <int FA, int FB, int NT>
__global__ void __launch_bounds__(128) qmv_kernel(const __grid_constant__ QmvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kGemvWarps * 4];
  pdl_launch_dependents();
  const int group = blockIdx.x, split = blockIdx.y;
  float acc[2][NT][4];
  if constexpr (FA == FB) {
    const int seg = group < p.seg[0].groups ? 0 : 1;
    gemv_segment<FA, NT>(p, p.seg[seg], seg ? group - p.seg[0].groups : group, split, smem, bars, acc);
  } else {
    if (group < p.seg[0].groups)
      gemv_segment<FA, NT>(p, p.seg[0], group, split, smem, bars, acc);
    else
      gemv_segment<FB, NT>(p, p.seg[1], group - p.seg[0].groups, split, smem, bars, acc);
  }
  reduce_and_epilogue<NT>(p, group, split, acc, reinterpret_cast<float*>(smem));
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
  uint8_t* out = tiles + (((size_t)(rt16 >> 1) * k_tiles + kt) * 2 + (rt16 & 1)) * TB;
  const int r0 = rt16 * 16;
  const int kbase = kt * KT;
  if (fmt == WF_BF16) {
    for (int s = 0; s < KT / 16; ++s) {
      uint16_t v[8];
      for (int p = 0; p < 8; ++p) {
        // a0: (g, 2t..2t+1), a1: (g+8, 2t..), a2: (g, 2t+8..), a3: (g+8, 2t+8..)
        const int reg = p >> 1, lo = p & 1;
        const int row = g + ((reg & 1) ? 8 : 0), col = 2 * t + ((reg & 2) ? 8 : 0) + lo;
        const uint8_t* src = raw + (size_t)(r0 + row) * row_bytes + (size_t)(kbase + 16 * s + col) * 2;
        v[p] = (uint16_t)(src[0] | (src[1] << 8));
      }
      uint32_t* dst = reinterpret_cast<uint32_t*>(out + s * 512 + lane * 16);
      for (int r = 0; r < 4; ++r) dst[r] = (uint32_t)v[2 * r] | ((uint32_t)v[2 * r + 1] << 16);
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
    uint32_t w = 0, hw = 0;
    for (int p = 0; p < 8; ++p) {
      int row, col;
      nib_pos(p, g, t, row, col);
      const uint8_t* rowp = raw + (size_t)(r0 + row) * row_bytes;
      const int k = kbase + 16 * s + col;
      w |= (uint32_t)code_at(rowp, fmt, k) << (4 * p);
      (void)hw;
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

template <int FA, int FB, int NT>
cudaError_t launch_inst(const QmvParams& p, cudaStream_t stream, bool pdl) {
  constexpr int ringA = kGemvWarps * fmt_stages(FA) * fmt_pair_bytes(FA);
  constexpr int ringB = kGemvWarps * fmt_stages(FB) * fmt_pair_bytes(FB);
  constexpr int ysb = kMaxRows * kGroupRows * 4;
  constexpr int smem = ringA > ringB ? (ringA > ysb ? ringA : ysb) : (ringB > ysb ? ringB : ysb);
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(qmv_kernel<FA, FB, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.seg[0].groups + p.seg[1].groups, p.S, 1);
  cfg.blockDim = dim3(kGemvWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qmv_kernel<FA, FB, NT>, p);
}

template <int FA, int FB>
cudaError_t launch_nt(const QmvParams& p, cudaStream_t s, bool pdl) {
  const int nt = (p.M + 7) / 8;
  if (nt <= 1) return launch_inst<FA, FB, 1>(p, s, pdl);
  if (nt <= 2) return launch_inst<FA, FB, 2>(p, s, pdl);
  if (nt <= 4) return launch_inst<FA, FB, 4>(p, s, pdl);
  return launch_inst<FA, FB, 8>(p, s, pdl);
}

}  // namespace

cudaError_t launch_qmv(const QmvParams& p, cudaStream_t s, bool pdl) {
  if (p.M < 1 || p.M > kMaxRows) return cudaErrorInvalidValue;
  const int fa = p.seg[0].fmt, fb = p.seg[1].groups ? p.seg[1].fmt : fa;
  if (fa == WF_Q4_K && fb == WF_Q4_K) return launch_nt<WF_Q4_K, WF_Q4_K>(p, s, pdl);
  if (fa == WF_Q4_K && fb == WF_Q6_K) return launch_nt<WF_Q4_K, WF_Q6_K>(p, s, pdl);
  if (fa == WF_Q6_K && fb == WF_Q6_K) return launch_nt<WF_Q6_K, WF_Q6_K>(p, s, pdl);
  if (fa == WF_Q5_K && fb == WF_Q5_K) return launch_nt<WF_Q5_K, WF_Q5_K>(p, s, pdl);
  if (fa == WF_Q8_0 && fb == WF_Q8_0) return launch_nt<WF_Q8_0, WF_Q8_0>(p, s, pdl);
  if (fa == WF_BF16 && fb == WF_BF16) return launch_nt<WF_BF16, WF_BF16>(p, s, pdl);
  return cudaErrorNotSupported;
}

cudaError_t launch_repack(const uint8_t* raw, int fmt, int N, int K, uint8_t* tiles, cudaStream_t s) {
  const int KT = fmt_kt(fmt);
  if (N % 32 || K % KT || fmt_tile_bytes(fmt) == 0) return cudaErrorInvalidValue;
  repack_kernel<<<dim3(N / 16, K / KT), 32, 0, s>>>(raw, fmt, N, K, tiles);
  return cudaGetLastError();
}

}  // namespace specb200
