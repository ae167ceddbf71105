"""Tensor-parallel host logic on the CPU: the receive-buffer handle exchange
over a gloo process group (world size 2 and 3), as every rank runs it before
its first forward."""

import json
import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(mode, out_dir, world, extra=(), timeout=300, env=None):
    """Starts `world` tp_worker.py ranks and waits for all of them (bounded)."""
    port = free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), mode, str(out_dir), str(r),
                               str(world), str(port), *extra], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(world)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=timeout)[0])
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} exited {p.returncode}:\n{outs[r][-3000:]}"


@pytest.mark.parametrize("world", [2, 3])
def test_handle_exchange_gloo(tmp_path, world):
    run_ranks("exchange", tmp_path, world)
    for r in range(world):
        with open(tmp_path / f"exchange_{r}.json") as f:
            d = json.load(f)
        assert d == {"ok": True, "n": world}


def test_connect_validates_before_any_device_call(pkg):
    """tp_connect on a non-tensor-parallel handle fails with the reference's
    Sampling/invalid error class and touches no device (null model here)."""
    import ctypes
    lib = ctypes.CDLL(pkg.LIB_PATH)
    lib.spec_tp_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.spec_tp_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.spec_tp_size.argtypes = [ctypes.c_void_p]
    buf = ctypes.create_string_buffer(64)
    assert lib.spec_tp_connect(None, buf, 2) == 1
    assert lib.spec_tp_handle(None, buf, 64) == -1
    assert lib.spec_tp_size(None) == 0
