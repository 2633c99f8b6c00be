"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, agrees with the oracle on the pure-host functions, fails
cleanly without a device, and its exp is glibc's expf bit for bit."""
import ctypes as C
import os
import re
import threading

import numpy as np
import pytest

from conftest import ROOT, hale_pkg
from oracle import oracle as O

HEADER = os.path.join(ROOT, "include", "hale_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(hale_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    hale = hale_pkg()
    L = hale.lib()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    # and the binding covers exactly the declared surface
    assert set(names) == set(hale.SIGNATURES)


def test_library_exports_nothing_undeclared():
    """Hidden visibility: only the C ABI is exported (checked with nm)."""
    import subprocess
    hale = hale_pkg()
    out = subprocess.run(["nm", "-D", "--defined-only", hale.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    hale_syms = {s for s in exported if s.startswith("hale_")}
    assert hale_syms == set(declared_functions())


@pytest.mark.parametrize("dtype", [O.F32, O.F16, O.BF16, O.Q8_0, O.Q4_0])
def test_row_bytes_agrees_with_the_reference_layout(dtype):
    """DType::row_bytes (dtype.rs:53-61)."""
    hale = hale_pkg()
    for cols in (0, 1, 13, 32, 33, 64, 2048, 14336):
        assert hale.row_bytes(dtype, cols) == O.row_bytes(dtype, cols), (dtype, cols)
    assert hale.row_bytes(9, 32) is None


def test_ctx_create_without_a_device_reports_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    hale = hale_pkg()
    h = C.c_void_p()
    st = hale.lib().hale_ctx_create(0, C.byref(h))
    assert st == hale.E_NO_DEVICE
    buf = C.create_string_buffer(256)
    assert hale.lib().hale_last_error(None, buf, 256) == hale.E_NO_DEVICE
    assert b"device" in buf.value


def test_device_exp_is_glibc_expf_for_every_float():
    """hale_expf (the exp every kernel uses) == libm expf over all 2^32 inputs.

    The oracle calls the platform libm, as Rust's f32::exp does on Linux, so
    this pins softmax / SiLU / sampling temperature to the reference."""
    hale = hale_pkg()
    chunk = 1 << 26
    bad = []

    def run(start):
        u = np.arange(start, start + chunk, dtype=np.uint64).astype(np.uint32)
        x = u.view(np.float32)
        a = hale.expf_host(x)
        b = O.expf_batch(x)
        ua, ub = a.view(np.uint32), b.view(np.uint32)
        nan = np.isnan(b) & np.isnan(a)
        diff = (ua != ub) & ~nan
        if diff.any():
            bad.append((start, int(np.flatnonzero(diff)[0])))

    starts = list(range(0, 1 << 32, chunk))
    threads = []
    for i in range(0, len(starts), 8):
        ts = [threading.Thread(target=run, args=(s,)) for s in starts[i:i + 8]]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        threads.extend(ts)
    assert not bad, bad[:4]


def test_null_handles_are_rejected_without_a_device():
    """Entry points given NULL handles answer HALE_E_INVALID_ARGUMENT (the
    reference's validation errors) before touching any device."""
    hale = hale_pkg()
    lib = hale.lib()
    n = C.c_uint32()
    params = hale.SamplingParams(0.0, 1.0, 0, 1.0)
    prompt = (C.c_uint32 * 2)(1, 2)
    out = (C.c_uint32 * 4)()
    st = lib.hale_decoder_generate(None, None, prompt, 2, C.byref(params), 42, 4, None, 0, out, C.byref(n),
                                   None, None, None)
    assert st == hale.E_INVALID_ARGUMENT
    assert lib.hale_decoder_set_comm(None, None) == hale.E_INVALID_ARGUMENT
    assert lib.hale_pool_set_source(None, None, None) == hale.E_INVALID_ARGUMENT
    assert lib.hale_moe_forward_ep(None, None, None, None, None, 0, None, None, None, None) == hale.E_INVALID_ARGUMENT
