"""unltd_gemv_noalloc: the GEMV for callers that cannot allocate GPU memory.

Such callers (code inside an allocator or memory pool, hosts that reserve all
device memory up front, code that must avoid cudaMalloc's implicit
synchronisation) get a variant whose scratch is a fixed array compiled into
the library. This test calls it through the C ABI and checks it against
unltd_gemv on two calls in a row (the array keeps the previous call's
contents, so the second call shows nothing stale leaks through), with the
same bars as the other GEMV tests: bit-identical in Q8K_EXACT mode, and in
F32X mode equal to unltd_gemv (same kernels) and within 1e-4 of the f64 truth.
Every case runs with an x the GEMV quantizes in its own prologue (16-byte
aligned) and with an x 4 bytes past a 16-byte boundary, which makes the prep
kernel build the x image in the fixed array.
It lives in its own file named to be collected last, and passes alone or
after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from __graft_entry__ import build

    build()
    torch.cuda.set_device(0)
    torch.cuda.set_stream(torch.cuda.Stream())
    c = ug.Context(0, stream=torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def _misaligned(x):
    """x on the device 4 bytes past a 16-byte boundary (prep-kernel path)."""
    buf = torch.zeros(x.size + 4, device="cuda")
    v = buf[1:1 + x.size]
    v.copy_(torch.from_numpy(x))
    assert v.data_ptr() % 16 == 4
    return v


def _noalloc(w, x, y, mode):
    s = torch.cuda.current_stream().cuda_stream
    rc = ug.lib().unltd_gemv_noalloc(w.h, x.data_ptr(), y.data_ptr(), mode, ctypes.c_void_p(s))
    if rc != 0:
        raise ug.UnltdError(rc, ug.last_error())


@pytest.mark.parametrize("aligned", [True, False], ids=["prologue", "prep"])
@pytest.mark.parametrize("dtype,dim_in,dim_out", [(ug.Q4K, 4096, 1000), (ug.Q6K, 12288, 300), (ug.Q8_0, 4096, 513)])
def test_noalloc_matches_gemv_twice(ctx, dtype, dim_in, dim_out, aligned):
    wb = synth.quant_weights(dtype, dim_in, dim_out, seed=77 + dim_out)
    w = ctx.upload(wb, dtype, dim_in, dim_out)
    modes = [ug.MODE_F32X] if dtype == ug.Q8_0 else [ug.MODE_Q8K, ug.MODE_F32X]
    for mode in modes:
        for call in range(2):  # two calls in a row, different inputs
            x = synth.activations(dim_in, seed=500 + call + (0 if aligned else 10))
            xd = torch.from_numpy(x).cuda() if aligned else _misaligned(x)
            y_ref = torch.empty(dim_out, device="cuda")
            y = torch.full((dim_out,), float("nan"), device="cuda")
            ctx.gemv(w, xd, y_ref, mode)
            _noalloc(w, xd, y, mode)
            torch.cuda.synchronize()
            a, b = y.cpu().numpy(), y_ref.cpu().numpy()
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (mode, call)
            if mode == ug.MODE_F32X:
                truth = oracle.gemv_quant_f64(x, wb, dim_in, dim_out, dtype, nthreads=8)
                assert np.max(np.abs(a - truth)) <= 1e-4 * np.max(np.abs(truth))
            else:
                ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, dtype, nthreads=8)
                assert np.array_equal(a.view(np.uint32), ref.view(np.uint32))
    w.free()


def test_noalloc_rejects_dim_in_beyond_limit(ctx):
    dim_in = 16384 + 256
    wb = synth.quant_weights(ug.Q4K, dim_in, 2, seed=3)
    w = ctx.upload(wb, ug.Q4K, dim_in, 2)
    x = torch.zeros(dim_in, device="cuda")
    y = torch.zeros(2, device="cuda")
    with pytest.raises(ug.UnltdError) as ei:
        _noalloc(w, x, y, ug.MODE_Q8K)
    assert ei.value.status == 4 and "16384" in str(ei.value)
    w.free()


def test_noalloc_on_two_devices():
    """Weights on devices 0 and 1 in one process: each device gets its own
    set-up (symbol address, kernel attributes) and the same bits as
    unltd_gemv there."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from __graft_entry__ import build

    build()
    dim_in, dim_out = 4096, 700
    wb = synth.quant_weights(ug.Q4K, dim_in, dim_out, seed=21)
    x = synth.activations(dim_in, seed=22)
    ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, ug.Q4K, nthreads=8)
    for dev in (0, 1):
        with torch.cuda.device(dev):
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                c = ug.Context(dev, stream=st.cuda_stream)
                w = c.upload(wb, ug.Q4K, dim_in, dim_out)
                for xd in (torch.from_numpy(x).cuda(), _misaligned(x)):
                    y = torch.full((dim_out,), float("nan"), device="cuda")
                    _noalloc(w, xd, y, ug.MODE_Q8K)
                    st.synchronize()
                    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), dev
                w.free()
                c.close()
