"""The C-ABI library loads, exports every symbol include/unltd_gpu.h declares,
and its argument checks (mirrors of the reference's asserts) answer without a
GPU. No compute call runs here."""
import os
import re

import numpy as np
import pytest

import unltd_gpu as ug

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    syms = set()
    for name in os.listdir(os.path.join(REPO, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(REPO, "include", name)).read()
            syms |= set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(unltd_[a-z_0-9]+)\s*\(", text, re.M))
    return syms


@pytest.fixture(scope="module")
def L():
    from __graft_entry__ import build

    build()
    return ug.lib()


def test_every_declared_symbol_is_exported(L):
    syms = _declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    bound = {n for n, _, _ in ug.SIGNATURES}
    assert syms <= bound, syms - bound


def test_rust_binding_declares_exported_symbols(L):
    """Every extern "C" function the Rust FFI crate (rust/unltd-tensor-gpu)
    declares is exported by the library and declared in the header, with the
    same number of parameters as the header's prototype."""
    src = open(os.path.join(REPO, "rust", "unltd-tensor-gpu", "src", "lib.rs")).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    decls = dict(re.findall(r"fn (unltd_[a-z_0-9]+)\(([^)]*)\)", block, re.S))
    assert {"unltd_gemv_quant", "unltd_gemv_quant_q8k", "unltd_dequantize_q4_k", "unltd_gemv"} <= set(decls)
    header = "".join(open(os.path.join(REPO, "include", n)).read() for n in os.listdir(os.path.join(REPO, "include"))
                     if n.endswith(".h"))
    for name, args in decls.items():
        assert hasattr(L, name), name
        m = re.search(r"\b%s\(([^)]*)\)" % name, header, re.S)
        assert m, name
        n_h = 0 if m.group(1).strip() in ("", "void") else m.group(1).count(",") + 1
        n_r = 0 if not args.strip() else args.count(",") + 1
        assert n_h == n_r, (name, n_h, n_r)


def test_row_bytes_match_reference_sizing(L):  # min_forward.rs:52-80
    assert ug.row_bytes(ug.F32, 4096) == 16384
    assert ug.row_bytes(ug.Q4K, 4096) == 16 * 144
    assert ug.row_bytes(ug.Q6K, 4096) == 16 * 210
    assert ug.row_bytes(ug.Q8_0, 64) == 2 * 34
    assert ug.row_bytes(ug.Q4K, 4097) == 0
    assert ug.row_bytes(ug.Q8_0, 33) == 0
    assert ug.row_bytes(ug.F16, 64) == 0


def test_abi_version(L):
    assert L.unltd_abi_version() == 1


def _expect(status, fn, *args):
    with pytest.raises(ug.UnltdError) as ei:
        fn(*args)
    assert ei.value.status == status, str(ei.value)


def test_host_api_refusals_mirror_reference_asserts(L):  # quants.rs:430-452, 482-505
    x = np.zeros(512, np.float32)
    w = np.zeros(2 * 144, np.uint8)
    out = np.zeros(2, np.float32)
    _expect(2, ug.gemv_quant, np.zeros(3, np.float32), x, w, 512, 2, ug.Q4K)    # len(out) != dim_out
    _expect(2, ug.gemv_quant, out, x[:256], w, 512, 2, ug.Q4K)                  # len(x) < dim_in
    _expect(3, ug.gemv_quant, out, x, w, 300, 2, ug.Q4K)                        # dim_in % 256
    _expect(2, ug.gemv_quant, out, x, w[:-1], 256, 2, ug.Q4K)                   # len(w)
    _expect(4, ug.gemv_quant, out, x, w, 256, 2, ug.F16)                        # dtype without kernel
    _expect(4, ug.gemv_quant_q8k, out, x, np.zeros(2 * 34 * 8, np.uint8), 256, 2, ug.Q8_0)  # no Q8_K dot
    _expect(2, ug.dequantize_q4_k, np.zeros(255, np.float32), np.zeros(144, np.uint8))


def test_no_device_is_an_error_not_a_fallback(L):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(ug.UnltdError) as ei:
        ug.Context(0)
    assert ei.value.status == 7  # NO_DEVICE
    # a well-formed host call must fail loudly too (no CPU path behind it)
    with pytest.raises(ug.UnltdError):
        ug.gemv_quant(np.zeros(1, np.float32), np.zeros(256, np.float32), np.zeros(144, np.uint8), 256, 1, ug.Q4K)
