"""A verify completes while an unrelated kernel holds half the SMs (GPU).

Inside one forward-kernel launch, chunks of a later op wait for the groups
that other CTAs of the same launch produce, so no such CTA may wait for a CTA
that has not started.  Multi-op launches therefore run cooperative (the
hardware starts the grid only when every CTA fits, and refuses a grid that
never could).

Here a kernel of the test's own (compiled with NVRTC; it spins on
%globaltimer for 3 s, so it always ends) takes the shared memory of 74 of the
148 SMs from another stream, and a verify of a 2-layer model with the
Llama-3-8B layer shapes (444-chunk ops) is issued on the decoder's stream
meanwhile.  Every device wait of the forward gives up after 2 s, so a forward
whose resident CTAs waited on CTAs that cannot start would fail with
SPEC_ERR_TIMEOUT.  It must instead return logits bit-identical to an
undisturbed run.
"""

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OCCUPY_SRC = rb"""
extern "C" __global__ void occupy(unsigned long long ns, int* done) {
  extern __shared__ unsigned char held[];
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  held[threadIdx.x] = (unsigned char)threadIdx.x;
  do {
    __nanosleep(2000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < ns);
  if (threadIdx.x == 0) atomicAdd(done, (int)held[0] + 1);
}
"""

LLAMA8B_2L = dict(arch="llama", n_layers=2, hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=128256,
                  rope_theta=5e5, eps=1e-5)


def _check(res):
    """cuda-python calls return (status, *values): assert success, return the value(s)."""
    if not isinstance(res, tuple):
        res = (res,)
    status = getattr(res[0], "value", res[0])
    assert status == 0, f"CUDA driver / NVRTC call failed: {res[0]}"
    return res[1] if len(res) == 2 else (res[1:] or None)


def _occupier():
    from cuda.bindings import driver as cu
    from cuda.bindings import nvrtc
    prog = _check(nvrtc.nvrtcCreateProgram(OCCUPY_SRC, b"occupy.cu", 0, [], []))
    opts = [b"--gpu-architecture=sm_100a"]
    res = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
    assert int(res[0]) == 0, "NVRTC compile of the occupying kernel failed"
    size = _check(nvrtc.nvrtcGetCUBINSize(prog))
    cubin = b" " * size
    _check(nvrtc.nvrtcGetCUBIN(prog, cubin))
    mod = _check(cu.cuModuleLoadData(cubin))
    fn = _check(cu.cuModuleGetFunction(mod, b"occupy"))
    return cu, fn


def test_verify_while_half_the_sms_are_held(pkg):
    import torch
    torch.cuda.init()
    dec = pkg.B200Decoder.synthetic(**LLAMA8B_2L, quant_mix="Q4_K_M", seed=5, max_ctx=512)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, LLAMA8B_2L["vocab"], size=64).tolist()
    drafts = rng.integers(0, LLAMA8B_2L["vocab"], size=4).tolist()
    dec.observe(prompt)
    want = dec.batched_logits(drafts)  # also captures the forward's CUDA graph
    dec.rollback_to(len(prompt))

    cu, fn = _occupier()
    props = torch.cuda.get_device_properties(0)
    n_sms = props.multi_processor_count
    smem = 227 * 1024  # one block per SM
    _check(cu.cuFuncSetAttribute(fn, cu.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, smem))
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    side = torch.cuda.Stream()
    blocks = n_sms // 2
    torch.cuda.synchronize()
    args = ((3_000_000_000, done.data_ptr()), (ctypes.c_ulonglong, ctypes.c_void_p))
    _check(cu.cuLaunchKernel(fn, blocks, 1, 1, 128, 1, 1, smem, cu.CUstream(side.cuda_stream), args, 0))
    time.sleep(0.2)  # the occupying blocks are resident before the verify is issued
    t0 = time.perf_counter()
    got = dec.batched_logits(drafts)
    elapsed = time.perf_counter() - t0
    side.synchronize()
    assert int(done.item()) == blocks, "the occupying kernel did not run to its end"
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"logits differ ({elapsed:.2f} s)"
    dec.close()
