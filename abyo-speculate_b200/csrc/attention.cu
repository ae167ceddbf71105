// Verify-step attention as standalone kernels: split-KV flash decode over the
// rollback KV cache (one CTA per (split, KV head)), then one warp per
// (KV head, row, 32 head columns) merging the splits into the O-projection
// operand.  The arithmetic lives in attn_core.cuh, shared with the attention
// ops of the persistent forward kernel; these kernels serve callers outside
// the forward (the EAGLE draft block) and the separate-kernel mode.
#include "common.cuh"
#include "kernels.cuh"
#include "attn_core.cuh"

namespace specb200 {

namespace {

// Up to two 16-row tiles (verify rows): 4 warps, warp pairs split the head
// columns (all four busy).  More tiles (tree verifies): 8 warps, one per
// tile, so a split's row tiles take half as many rounds and twice the warps
// hide each other's latency (S is formed once per tile either way).
template <int HD, bool BF16, int W>
__global__ void __launch_bounds__(W * 32) attn_split_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  pdl_launch_dependents();
  if constexpr (W == 4)
    attn::split_unit<HD, BF16, 2, 4>(p, blockIdx.x, blockIdx.y, smem_raw, p.chunk, [] { pdl_wait(); });
  else
    attn::split_unit<HD, BF16, 1, W>(p, blockIdx.x, blockIdx.y, smem_raw, p.chunk, [] { pdl_wait(); });
}

// 64 registers (8 CTAs per SM): tree verifies have thousands of merge items.
template <int HD>
__global__ void __launch_bounds__(128, 8) attn_combine_kernel(const __grid_constant__ AttnParams p, int nt_total) {
  pdl_launch_dependents();
  pdl_wait();
  attn::combine_item<HD>(p, nt_total, blockIdx.x * 4 + (threadIdx.x >> 5), threadIdx.x & 31);
}

template <int HD, bool BF16, int W>
cudaError_t launch_split(const AttnParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = attn::unit_smem_bytes(HD, p.chunk, W);
  static size_t attr = 0;  // largest dynamic shared memory granted so far (chunk sizes differ per caller)
  if (smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<HD, BF16, W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    attr = smem;
  }
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, p.n_kv, 1);
  cfg.blockDim = dim3(W * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_split_kernel<HD, BF16, W>, p);
}

template <int HD, bool BF16>
cudaError_t launch_hd(const AttnParams& p, int nt, cudaStream_t s, bool pdl) {
  cudaError_t e = p.M * p.G <= 32 ? launch_split<HD, BF16, 4>(p, s, pdl) : launch_split<HD, BF16, 8>(p, s, pdl);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  const int items = attn_combine_items(p.n_kv, p.M * p.G, HD);
  cudaLaunchConfig_t cfg2 = {};
  cfg2.gridDim = dim3((items + 3) / 4, 1, 1);
  cfg2.blockDim = dim3(128, 1, 1);
  cfg2.dynamicSmemBytes = 0;
  cfg2.stream = s;
  cfg2.attrs = at;
  cfg2.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg2, attn_combine_kernel<HD>, p, nt);
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, int nt, cudaStream_t s, bool pdl) {
  if (p.M < 1 || p.M > kMaxRows || p.chunk % attn::kKeyBlock) return cudaErrorInvalidValue;
  if (p.hd == 128) return p.act_bf16 ? launch_hd<128, true>(p, nt, s, pdl) : launch_hd<128, false>(p, nt, s, pdl);
  if (p.hd == 64) return p.act_bf16 ? launch_hd<64, true>(p, nt, s, pdl) : launch_hd<64, false>(p, nt, s, pdl);
  return cudaErrorNotSupported;
}

}  // namespace specb200
