// spec_qmatmul_noalloc: the standalone dequant-matmul with every piece of
// per-call scratch in one file-scope device array, so a call allocates no
// memory.  The array is shared by all calls on a device; see the contract in
// include/spec_b200.h.
#include <atomic>

#include "../../include/spec_b200.h"
#include "common.cuh"
#include "model.h"

namespace specb200 {
namespace {

constexpr size_t kNoAllocBytes = SPEC_NOALLOC_SCRATCH_BYTES;
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;

// The scratch itself: operand fragments and column sums, split-K partials,
// split-K arrival counters, the op descriptor and its completion counter.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch per device, looked up once.
std::atomic<uint8_t*> g_scratch_ptr[kMaxDevices];

static_assert(sizeof(FwdOp) <= 1024, "descriptor slot too small");

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Byte offsets of one call's pieces inside the scratch.
struct Layout {
  size_t desc, done, counters, frag, x16, x32, part, total;
  size_t zero_begin, zero_end;  // [counters + done] must be zero at launch
};

Layout plan(int K, int nt, int groups, int chunks) {
  Layout L;
  size_t o = 0;
  L.desc = o;
  o += 1024;
  L.zero_begin = o;
  L.done = o;
  o += kAlign;
  L.counters = o;
  o = align_up(o + (size_t)groups * 4);
  L.zero_end = o;
  L.frag = o;
  o = align_up(o + (size_t)K * 8 * nt * 2);
  L.x16 = o;
  o = align_up(o + (size_t)(K / 16) * 8 * nt * 4);
  L.x32 = o;
  o = align_up(o + (size_t)(K / 32) * 8 * nt * 4);
  L.part = o;
  if (chunks > 1) o = align_up(o + (size_t)(chunks + groups) * kGroupRows * 8 * nt * 4);
  L.total = o;
  return L;
}

// Writes the by-value descriptor into the scratch slot on the stream, so the
// call needs no host staging buffer.
__global__ void noalloc_store_op_kernel(const __grid_constant__ FwdOp op, FwdOp* dst) {
  constexpr int words = (int)(sizeof(FwdOp) / sizeof(int4));
  const int4* src = reinterpret_cast<const int4*>(&op);
  int4* d = reinterpret_cast<int4*>(dst);
  for (int i = threadIdx.x; i < words; i += blockDim.x) d[i] = src[i];
}

// Setup, once per device, with that device current.
int scratch_for_device(int device, uint8_t** out) {
  if (device < 0 || device >= kMaxDevices) {
    set_thread_error("spec_qmatmul_noalloc: device ordinal out of range");
    return SPEC_ERR_INVALID;
  }
  uint8_t* p = g_scratch_ptr[device].load(std::memory_order_acquire);
  if (!p) {
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_thread_error("spec_qmatmul_noalloc: cudaGetSymbolAddress of the scratch array failed");
      return SPEC_ERR_CUDA;
    }
    g_scratch_ptr[device].store(p, std::memory_order_release);
  }
  *out = p;
  return SPEC_OK;
}

}  // namespace
}  // namespace specb200

using namespace specb200;

extern "C" int spec_qmatmul_noalloc(spec_qweight* w, const float* x_dev, int M, float* y_dev, void* stream) {
  if (!w || !x_dev || !y_dev || M < 1 || M > kMaxRows) {
    set_thread_error("spec_qmatmul_noalloc: null argument or M outside [1, 64]");
    return SPEC_ERR_INVALID;
  }
  QmatmulLaunch q;
  if (!qweight_launch_desc(w, M, y_dev, &q)) return SPEC_ERR_INVALID;
  // The weight's device is current for the call; the caller's comes back on return.
  DeviceGuard dg(q.device);
  {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != q.device) {
      set_thread_error("spec_qmatmul_noalloc: cudaSetDevice failed");
      return SPEC_ERR_CUDA;
    }
  }
  const int nt = nt_for_rows(M);
  const int groups = q.p.seg[0].groups + q.p.seg[1].groups;
  const Layout L = plan(q.p.K, nt, groups, q.p.chunks);
  if (L.total > kNoAllocBytes) {
    set_thread_error(
        "spec_qmatmul_noalloc: this shape needs more scratch than SPEC_NOALLOC_SCRATCH_BYTES "
        "(operand plus split-K partials); use spec_qmatmul");
    return SPEC_ERR_INVALID;
  }
  uint8_t* base = nullptr;
  int rc = scratch_for_device(q.device, &base);
  if (rc != SPEC_OK) return rc;

  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : q.stream;
  FwdOp op;
  op.q = q.p;
  op.q.part = reinterpret_cast<float*>(base + L.part);
  op.q.counters = reinterpret_cast<int*>(base + L.counters);
  op.q.xfrag = reinterpret_cast<const uint32_t*>(base + L.frag);
  op.q.xsum16 = reinterpret_cast<const float*>(base + L.x16);
  op.q.xsum32 = reinterpret_cast<const float*>(base + L.x32);
  op.dep = -1;

  cudaError_t e = cudaMemsetAsync(base + L.zero_begin, 0, L.zero_end - L.zero_begin, s);
  // The weight's 16-byte error word starts clear, so a synchronous call
  // reports only its own launch.
  if (e == cudaSuccess) e = cudaMemsetAsync(q.p.err, 0, 16, s);
  if (e == cudaSuccess)
    e = launch_make_operand(x_dev, M, q.p.K, nt, reinterpret_cast<uint32_t*>(base + L.frag),
                            reinterpret_cast<float*>(base + L.x16), reinterpret_cast<float*>(base + L.x32),
                            q.p.act_bf16, s);
  if (e == cudaSuccess) {
    noalloc_store_op_kernel<<<1, 32, 0, s>>>(op, reinterpret_cast<FwdOp*>(base + L.desc));
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    FwdParams fp;
    fp.ops = reinterpret_cast<const FwdOp*>(base + L.desc);
    fp.n_ops = 1;
    fp.done = reinterpret_cast<int*>(base + L.done);
    fp.err = q.p.err;
    fp.l2_ahead = q.l2_ahead;
    e = launch_fwd(fp, q.fmt_set, M, s, false);
  }
  if (e != cudaSuccess) {
    set_thread_error("spec_qmatmul_noalloc: CUDA launch failed");
    return SPEC_ERR_CUDA;
  }
  if (!stream) {
    // Synchronous call: a bounded wait inside the kernel that gave up left y
    // incomplete; that is reported here (and the word cleared).
    char msg[256];
    const int rc2 = take_device_error(q.p.err, s, msg, sizeof msg);
    if (rc2 != SPEC_OK) {
      set_thread_error(msg);
      return rc2;
    }
  }
  return SPEC_OK;
}
