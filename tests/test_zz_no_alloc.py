"""jv_qmatvec_noalloc (fixed device scratch, no allocation) against jv_qmatvec.

Collected last on purpose: it must pass both in a fresh process (first call on the device
does the scratch set-up) and after every other test has used the device.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

def _inputs(qtype, rows, cols, seed):
    import torch

    from jevstral_b200 import quant
    from jevstral_b200.synth import synth_normal, synth_quantize

    raw = synth_quantize(synth_normal(seed, rows, rows * cols, 0.02), qtype)
    dev = torch.device("cuda:0")
    d_raw = torch.from_numpy(raw).to(dev)
    tiled = torch.empty(quant.qweight_bytes(qtype, rows, cols), dtype=torch.uint8, device=dev)
    quant.qweight_pack(qtype, d_raw.data_ptr(), rows, cols, tiled.data_ptr())
    torch.cuda.synchronize()
    return tiled


@pytest.mark.parametrize("qtype,rows,cols", [("Q8_0", 3072, 3072), ("Q4_0", 9216, 3072), ("Q5_1", 3072, 9216)])
def test_noalloc_matches_qmatvec_on_two_calls_in_a_row(qtype, rows, cols):
    import torch

    from jevstral_b200 import quant
    from jevstral_b200._lib import check, lib

    tiled = _inputs(qtype, rows, cols, 17)
    rng = np.random.default_rng(rows ^ cols)
    t = quant.TYPE_IDS[qtype]
    outs = []
    # Two calls with the same input, then one with another: the two entry points pick the same
    # splits and run the same two kernels in the same order, so their outputs match bit for bit;
    # the third call must change the output, so a stale scratch value cannot pass.
    xs = [rng.uniform(-2, 2, cols).astype(np.float32)] * 2 + [rng.uniform(-2, 2, cols).astype(np.float32)]
    for call, xh in enumerate(xs):
        x = torch.from_numpy(xh).cuda()
        want = torch.empty(rows, dtype=torch.float32, device="cuda")
        got = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        check(lib.jv_qmatvec(t, tiled.data_ptr(), rows, cols, x.data_ptr(), want.data_ptr(), None))
        check(lib.jv_qmatvec_noalloc(t, tiled.data_ptr(), rows, cols, x.data_ptr(), got.data_ptr(), None))
        torch.cuda.synchronize()
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}"
        assert g.tobytes() == w.tobytes(), (call, float(np.abs(g - w).max()))
        outs.append(g)
    assert outs[0].tobytes() == outs[1].tobytes()
    assert not np.array_equal(outs[2], outs[1])


def test_noalloc_rejects_requests_beyond_the_scratch():
    """rows x splits above JV_QMATVEC_SCRATCH_FLOATS_MAX is refused on the host before anything is
    launched: the library's launch counter does not move and no CUDA error is left pending."""
    import torch

    from jevstral_b200._lib import JV_ERR_RANGE, lib

    rows, cols = 262144 + 128, 64  # one k step -> one split -> 262272 partials > 262144
    buf = torch.zeros(64, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    before = lib.jv_kernel_launches()
    rc = lib.jv_qmatvec_noalloc(8, buf.data_ptr(), rows, cols, buf.data_ptr(), buf.data_ptr(), None)
    assert rc == JV_ERR_RANGE
    assert b"scratch" in lib.jv_last_error()
    assert lib.jv_kernel_launches() == before
    torch.cuda.synchronize()  # raises if the call had left an asynchronous error behind
    assert torch.cuda.is_available() and float(buf.sum().item()) == 0.0
