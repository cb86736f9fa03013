"""Moving tensors between the reference's CPU carrier and the CUDA carrier
(``sw.move``), and DLPack import / export of CUDA-carrier tensors.

The move tests follow the behaviour the reference pins for its own bulk
moves (tests/test_move.py): values arrive, the source is released, layouts
(broadcast ones included) are kept, and gradients flow back across the
carrier boundary to the source's class.
"""

from __future__ import annotations

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, DType, Layout, Shape, Stride, Swizzle, SwizzleStage, Tensor  # noqa: E402

pytestmark = pytest.mark.gpu


def cpu_tensor(values, dtype=DType.Float32):
    t = Tensor(CPU(len(values), dtype=dtype), 0, Layout(Shape(len(values)), Stride(1)))
    for i, v in enumerate(values):
        t[i] = v
    return t


def values_of(t):
    return [t[i] for i in range(t.size())]


def test_move_cpu_to_cuda_copies_and_releases_the_source():
    from strideweave_b200 import CUDA
    from strideweave_b200.move import CpuToCudaMoveOperation

    src = cpu_tensor([1.5, -2.0, 3.25, 7.0])
    moved = sw.move(src, CUDA(4))
    assert type(moved.carrier) is CUDA
    assert values_of(moved) == [1.5, -2.0, 3.25, 7.0]
    assert src.carrier.is_released()
    assert type(moved.autograd_ctx) is CpuToCudaMoveOperation
    assert moved.autograd_ctx.inputs() == (src,)


def test_move_sizes_an_empty_cuda_destination_and_keeps_int32():
    from strideweave_b200 import CUDA

    src = cpu_tensor([3, -1, 2**30, 7], dtype=DType.Int32)
    with sw.no_grad():
        moved = sw.move(src, CUDA(0, dtype=DType.Int32))
    assert moved.autograd_ctx is None
    assert moved.carrier.size() == 4
    np.testing.assert_array_equal(moved.carrier.to_numpy(), [3, -1, 2**30, 7])


def test_round_trip_through_cuda_backpropagates_to_the_cpu_leaf():
    from strideweave_b200 import CUDA

    src = cpu_tensor([1.0, 2.0, 3.0])
    on_gpu = sw.move(src, CUDA(3))
    back = sw.move(on_gpu, CPU(3, dtype=DType.Float32))
    assert type(back.carrier) is CPU
    assert values_of(back) == [1.0, 2.0, 3.0]
    back.backward(cpu_tensor([10.0, 11.0, 12.0]))
    assert src.grad is not None
    assert type(src.grad.carrier) is CPU
    assert values_of(src.grad) == pytest.approx([10.0, 11.0, 12.0])


def test_broadcast_layout_moves_its_physical_span_only():
    from strideweave_b200 import CUDA

    lay = Layout(Shape([3, 4]), Stride([1, 0]))  # a column repeated four times
    src = Tensor(CPU(3, dtype=DType.Float32), 0, lay)
    for i, v in enumerate([2.0, 5.0, 7.0]):
        src.carrier.set_value(i, v)
    moved = sw.move(src, CUDA(0))
    assert moved.layout == lay
    assert moved.carrier.size() == 3
    assert [moved[i, j] for i in range(3) for j in range(4)] == [2.0] * 4 + [5.0] * 4 + [7.0] * 4


def test_move_into_and_out_of_a_swizzled_cuda_carrier():
    from strideweave_b200 import CUDA

    n = 256
    values = np.arange(n, dtype=np.float32) * 0.5 - 3.0
    swz = Swizzle(Shape(n), SwizzleStage(bits=2, base=2, shift=3))
    src = Tensor(CPU(n, dtype=DType.Float32), 0, Layout(Shape(n), Stride(1)))
    for i, v in enumerate(values):
        src.carrier.set_value(i, float(v))
    moved = sw.move(src, CUDA(n, swizzle=swz))
    np.testing.assert_array_equal(moved.carrier.to_numpy(), values)
    raw = moved.carrier.raw_numpy().view(np.float32)
    assert not np.array_equal(raw, values)  # stored permuted
    back = sw.move(moved, CPU(n, dtype=DType.Float32))
    assert values_of(back) == values.tolist()


# ---- DLPack ---------------------------------------------------------------------------


def test_import_a_torch_tensor_without_a_copy():
    torch = pytest.importorskip("torch")
    from strideweave_b200 import CUDA
    from strideweave_b200.dlpack import from_dlpack

    src = torch.arange(24, dtype=torch.float32, device="cuda").reshape(4, 6)
    t = from_dlpack(src)
    assert type(t.carrier) is CUDA
    assert t.carrier.data_ptr == src.data_ptr()
    assert [t[i, j] for i in range(4) for j in range(6)] == src.flatten().tolist()
    # the carrier reduces it in place ...
    row_max = sw.reduce_max(t, "a b -> a")
    np.testing.assert_array_equal(row_max.carrier.to_numpy(), src.max(dim=1).values.cpu().numpy())
    # ... and its writes land in the producer's memory
    t[1, 2] = -100.0
    torch.cuda.synchronize()
    assert src[1, 2].item() == -100.0


def test_import_strided_and_narrow_dtypes():
    torch = pytest.importorskip("torch")
    from strideweave_b200.dlpack import from_dlpack

    base = torch.randn(8, 16, device="cuda")
    view = base.t()  # strides (1, 16)
    t = from_dlpack(view)
    assert t.layout == Layout(Shape([16, 8]), Stride([1, 16]))
    assert [t[i, j] for i in range(16) for j in range(8)] == view.flatten().tolist()
    bf = torch.randn(32, device="cuda").to(torch.bfloat16)
    tb = from_dlpack(bf)
    assert tb.carrier.dtype().name == "BFloat16"
    np.testing.assert_array_equal(tb.carrier.to_numpy(), bf.float().cpu().numpy())
    f8 = torch.randn(32, device="cuda").to(torch.float8_e4m3fn)
    t8 = from_dlpack(f8)
    assert t8.carrier.dtype() is DType.E4M3
    np.testing.assert_array_equal(t8.carrier.to_numpy(), f8.float().cpu().numpy())


def test_export_mx_planes_and_bf16_to_torch():
    torch = pytest.importorskip("torch")
    from strideweave_b200 import CUDA
    from strideweave_b200.dlpack import DLPackExport

    vals = np.array([0.5, -1.5, 448.0, -0.0, 2.0, 3.0, -6.0, 0.25], dtype=np.float32)
    for dtype, torch_dtype in ((DType.E4M3, torch.float8_e4m3fn), (DType.E2M1, None),
                               (DType.Float32, torch.float32)):
        v = vals if dtype is not DType.E2M1 else np.array([0.5, -1.5, 6.0, -0.0, 2.0, 3.0, -6.0, 1.0], np.float32)
        c = CUDA(len(v), dtype=dtype)
        for i, x in enumerate(v):
            c.set_value(i, float(x))
        t = Tensor(c, 0, Layout(Shape(len(v)), Stride(1)))
        out = torch.from_dlpack(DLPackExport(t))
        assert out.data_ptr() == c.data_ptr
        if dtype is DType.E2M1:
            assert out.dtype == torch.float4_e2m1fn_x2 and out.numel() == len(v) // 2
            np.testing.assert_array_equal(out.view(torch.uint8).cpu().numpy(), c.raw_numpy())
        else:
            assert out.dtype == torch_dtype
            np.testing.assert_array_equal(out.float().cpu().numpy(), c.to_numpy())


def test_export_a_strided_view_and_keep_the_carrier_alive():
    torch = pytest.importorskip("torch")
    from strideweave_b200 import CUDA
    from strideweave_b200.dlpack import DLPackExport

    x = np.arange(12, dtype=np.float32)
    c = CUDA.from_numpy(x)
    t = Tensor(c, 1, Layout(Shape([3, 2]), Stride([4, 1])))  # offset 1, rows 4 apart
    out = torch.from_dlpack(DLPackExport(t))
    del t, c  # the exported capsule keeps the storage alive
    assert out.shape == (3, 2) and out.stride() == (4, 1)
    np.testing.assert_array_equal(out.cpu().numpy(), [[1, 2], [5, 6], [9, 10]])
