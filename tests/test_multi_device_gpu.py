"""One process driving two GPUs: a context on each of devices 0 and 1, the
tensor-core GEMV (Q8K_EXACT, > 48 KiB of shared memory per CTA) and the
tcgen05 GEMM on both, each device with its own kernel attributes. Plain
single-device work on each GPU; nothing crosses between them."""
import numpy as np
import pytest

import oracle
import synth
import unltd_gpu as ug

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_gemv_and_gemm_on_two_devices():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from __graft_entry__ import build

    build()
    dim_in, dim_out, m = 4096, 512, 64
    wb = synth.quant_weights(ug.Q4K, dim_in, dim_out, seed=31)
    x = synth.activations(dim_in, seed=32)
    X = synth.activations(dim_in, seed=33, rows=m)
    ref = oracle.gemv_quant_q8k(x, wb, dim_in, dim_out, ug.Q4K, nthreads=8)
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                c = ug.Context(dev, stream=st.cuda_stream)
                w = c.upload(wb, ug.Q4K, dim_in, dim_out)
                y = torch.full((dim_out,), float("nan"), device="cuda")
                c.gemv(w, torch.from_numpy(x).cuda(), y, ug.MODE_Q8K)
                Y = torch.full((m, dim_out), float("nan"), device="cuda")
                c.gemm(w, torch.from_numpy(X).cuda(), Y, m)
                c.synchronize()
                assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), dev
                outs.append(Y.cpu().numpy())
                w.free()
                c.close()
    assert np.all(np.isfinite(outs[0]))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
