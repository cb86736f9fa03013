"""The two-way MX quantiser (``sw_mx_quantize_dual``): one read of S gives the
planes blocked along its columns and along its rows.

* S = x: both planes bit for bit against the CPU restatement of OCP MX v1.0
  (x and x transposed).
* S = gelu(x) and S = x * gelu'(h): both planes bit for bit against the
  separate sequence (``sw_elementwise_f32``, then the oracle quantiser on its
  output).
* At a full MLP size (8192 x 4096): the same equality against the device's
  own separate kernels.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from strideweave_b200 import _native as N
from strideweave_b200 import kernels
from tests.gpu_util import empty, to_device, to_host
from tests.test_gpu_mx import adversarial

pytestmark = pytest.mark.gpu


def scale_bytes(n: int, k: int, layout: int) -> int:
    return O.scale_bytes_tc128(n, k // 32) if layout == N.SW_SCALES_TC128 else n * (k // 32)


def run_dual(fmt, xf, x_store, h_store, rows, cols, ld, layout, *, want_r=True, want_c=True):
    """Planes of S[rows, cols] read from row-pitch-`ld` stores; (payload, scales) or None each."""
    dx = to_device(x_store)
    dh = to_device(h_store) if h_store is not None else None
    rb = cols if fmt == O.E4M3 else cols // 2
    cb = rows if fmt == O.E4M3 else rows // 2
    bufs = {}
    if want_r:
        bufs["r"] = (empty(rows * rb, fill=0), empty(scale_bytes(rows, cols, layout), fill=0))
    if want_c:
        bufs["c"] = (empty(cols * cb, fill=0), empty(scale_bytes(cols, rows, layout), fill=0))
    r = bufs.get("r")
    c = bufs.get("c")
    N.check(N.lib.sw_mx_quantize_dual(
        fmt, xf, N.c_void_p(dx.ptr), N.c_void_p(dh.ptr if dh else None), rows, cols, ld,
        N.c_void_p(r[0].ptr if r else None), rb, N.c_void_p(r[1].ptr if r else None), layout, cols // 32,
        N.c_void_p(c[0].ptr if c else None), cb, N.c_void_p(c[1].ptr if c else None), layout, rows // 32, None))
    out = {}
    if r:
        s = to_host(r[1], scale_bytes(rows, cols, layout), np.uint8)
        out["r"] = (to_host(r[0], (rows, rb), np.uint8),
                    s.reshape(rows, cols // 32) if layout == N.SW_SCALES_ROWMAJOR else s)
    if c:
        s = to_host(c[1], scale_bytes(cols, rows, layout), np.uint8)
        out["c"] = (to_host(c[0], (cols, cb), np.uint8),
                    s.reshape(cols, rows // 32) if layout == N.SW_SCALES_ROWMAJOR else s)
    return out


def padded(a: np.ndarray, ld: int) -> np.ndarray:
    store = np.full((a.shape[0], ld), np.float32(7.5))  # the pitch padding must not be read
    store[:, : a.shape[1]] = a
    return store


def assert_planes(got, fmt, S, layout):
    for key, m in (("r", S), ("c", np.ascontiguousarray(S.T))):
        if key not in got:
            continue
        pw, sw_ = O.mx_quantize(fmt, m, scale_layout=layout)
        np.testing.assert_array_equal(got[key][1], sw_, err_msg=f"{key} scales")
        np.testing.assert_array_equal(got[key][0], pw, err_msg=f"{key} payload")


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("layout", [N.SW_SCALES_ROWMAJOR, N.SW_SCALES_TC128])
@pytest.mark.parametrize("rows,cols,ld", [(32, 128, 128), (96, 384, 388), (256, 1024, 1024), (160, 256, 260)])
def test_plain_planes_match_the_oracle(fmt, layout, rows, cols, ld):
    x = adversarial(rows, cols, seed=rows + cols)
    got = run_dual(fmt, N.SW_XF_NONE, padded(x, ld), None, rows, cols, ld, layout)
    assert_planes(got, fmt, x, layout)


def separate_elementwise(op, x, h):
    """S from the device's elementwise kernel (the unfused sequence's first step)."""
    n = x.size
    a = to_device(h if op == N.SW_EW_GELU_GRAD else x)
    b = to_device(x) if op == N.SW_EW_GELU_GRAD else None
    out = empty(4 * n)
    N.check(N.lib.sw_elementwise_f32(op, n, N.c_void_p(a.ptr), N.c_void_p(b.ptr if b else None),
                                     N.c_void_p(out.ptr), 0.0, None))
    return to_host(out, x.shape, np.float32)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("xf,op", [(N.SW_XF_GELU, N.SW_EW_GELU), (N.SW_XF_GELU_GRAD, N.SW_EW_GELU_GRAD)])
def test_gelu_planes_equal_the_separate_sequence(fmt, xf, op):
    rows, cols = 128, 512
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    h = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    x[5, :32] = 0.0
    x[6, 40] = np.nan
    h[7, 70] = np.inf
    x[9, 100] = -np.inf
    S = separate_elementwise(op, x, h if xf == N.SW_XF_GELU_GRAD else None)
    got = run_dual(fmt, xf, x, h if xf == N.SW_XF_GELU_GRAD else None, rows, cols, cols, N.SW_SCALES_TC128)
    assert_planes(got, fmt, S, N.SW_SCALES_TC128)


@pytest.mark.parametrize("want_r,want_c", [(True, False), (False, True)])
def test_one_plane_pair_only(want_r, want_c):
    x = adversarial(64, 256, seed=3)
    got = run_dual(O.E4M3, N.SW_XF_NONE, x, None, 64, 256, 256, N.SW_SCALES_TC128, want_r=want_r, want_c=want_c)
    assert ("r" in got) == want_r and ("c" in got) == want_c
    assert_planes(got, O.E4M3, x, N.SW_SCALES_TC128)


def test_untileable_shapes_are_refused():
    x = to_device(np.zeros((64, 256), np.float32))
    p = empty(64 * 256)
    s = empty(O.scale_bytes_tc128(64, 8))
    for rows, cols, ld in ((33, 256, 256), (64, 200, 256), (64, 128, 130)):
        with pytest.raises(NotImplementedError):
            N.check(N.lib.sw_mx_quantize_dual(O.E4M3, N.SW_XF_NONE, N.c_void_p(x.ptr), None, rows, cols, ld,
                                              N.c_void_p(p.ptr), cols, N.c_void_p(s.ptr), N.SW_SCALES_TC128,
                                              0, None, 0, None, N.SW_SCALES_TC128, 0, None))
    with pytest.raises(ValueError):  # GELU' without the pre-activation
        N.check(N.lib.sw_mx_quantize_dual(O.E4M3, N.SW_XF_GELU_GRAD, N.c_void_p(x.ptr), None, 64, 256, 256,
                                          N.c_void_p(p.ptr), 256, N.c_void_p(s.ptr), N.SW_SCALES_TC128, 0,
                                          None, 0, None, N.SW_SCALES_TC128, 0, None))


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_full_size_gelu_grad_equals_the_device_sequence(fmt):
    """8192 x 4096 (an MLP hidden activation): dual planes == elementwise
    kernel + two sw_mx_quantize calls, compared on the host byte for byte."""
    import torch

    rows, cols = 4096, 8192  # memory rows = hidden features, columns = batch
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    h = torch.randn(rows, cols, device="cuda", generator=g) * 2
    rb, cb = (cols, rows) if fmt == O.E4M3 else (cols // 2, rows // 2)
    outs = {}
    for path in ("dual", "separate"):
        pr = torch.zeros(rows * rb, dtype=torch.uint8, device="cuda")
        sr = torch.zeros(O.scale_bytes_tc128(rows, cols // 32), dtype=torch.uint8, device="cuda")
        pc = torch.zeros(cols * cb, dtype=torch.uint8, device="cuda")
        sc = torch.zeros(O.scale_bytes_tc128(cols, rows // 32), dtype=torch.uint8, device="cuda")
        if path == "dual":
            kernels.mx_quantize_dual(fmt, N.SW_XF_GELU_GRAD, x.data_ptr(), h.data_ptr(), rows, cols, cols,
                                     (pr.data_ptr(), sr.data_ptr()), (pc.data_ptr(), sc.data_ptr()))
        else:
            s = torch.empty_like(x)
            N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU_GRAD, x.numel(), N.c_void_p(h.data_ptr()),
                                             N.c_void_p(x.data_ptr()), N.c_void_p(s.data_ptr()), 0.0, None))
            kernels.mx_quantize(fmt, s.data_ptr(), rows, cols, cols, 1, pr.data_ptr(), rb, sr.data_ptr())
            kernels.mx_quantize(fmt, s.data_ptr(), cols, rows, 1, cols, pc.data_ptr(), cb, sc.data_ptr())
        torch.cuda.synchronize()
        outs[path] = [t.cpu().numpy() for t in (pr, sr, pc, sc)]
    for a, b in zip(outs["dual"], outs["separate"]):
        np.testing.assert_array_equal(a, b)
