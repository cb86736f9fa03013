"""The CPU oracle, pinned before it is trusted (no GPU needed).

Reductions and matmul are pinned bit-for-bit against outputs of the reference
CPU carrier (``tests/golden/*.npz``, made by ``tests/golden/make_golden.py``).
The MX quantiser has no reference counterpart: it is pinned by exhaustive
element-code round trips, hand-computed known answers for every rule the
project fixes (rounding ties, saturation, zero / NaN / Inf blocks, subnormal
block maxima) and by torch's float8_e4m3fn rounding for in-range values.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def red():
    return np.load(GOLDEN / "reductions.npz")


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32)


N, M = 64, 96
LAYOUTS = {
    "a": ("rowmajor", [(N, M)], [(M, 1)]),
    "b": ("colmajor", [(N, 1)], [(M, N)]),
    "c": ("tiled", [(16, 32), (N // 16, 16 * 32 * (M // 32))], [(32, 1), (M // 32, 16 * 32)]),
}


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
def test_reductions_match_reference_bit_for_bit(red, case, kind):
    storage_key, kept, reduced = LAYOUTS[case]
    got = O.reduce(kind, red[storage_key], 0, kept, reduced)
    want = red[f"{case}_{kind}"]
    if kind == "sum":
        # NaN payloads of a sum are unspecified (IEEE 754 6.2.3): equal where
        # finite, NaN where the reference is NaN.
        np.testing.assert_array_equal(got, want)
    else:
        np.testing.assert_array_equal(bits(got), bits(want))


def test_reference_pins_extrema_rules(red):
    mx = red["a_max"]
    assert bits(mx)[1] == 0x7FC00001  # first NaN payload wins
    assert bits(mx)[2] == 0x00000000  # all -0: two zeros give +0
    assert bits(mx)[3] == 0x80000000  # a single -0 keeps its sign
    assert bits(mx)[4] == 0x00000000
    am = red["a_argmax"]
    assert am[1] == 5 and am[5] == 3 and am[7] == 2 and am[8] == 0 and am[6] == 0


def test_swizzle_restatement_matches_reference_map(red):
    stages = [(3, 2, 3)]
    got = np.array([O.swizzle_index(int(i), stages) for i in red["swz_in"]])
    np.testing.assert_array_equal(got, red["swz_out"])


def test_swizzled_storage_reduces_like_logical_data(red):
    # A carrier that stores flat index f at swizzle(f): reading through the
    # swizzle must give the reference answer of the logical data.
    stages = [(3, 2, 3)]
    logical = np.zeros(8192, dtype=np.float32)
    logical[: N * M] = red["rowmajor"]
    physical = np.empty_like(logical)
    for f in range(8192):
        physical[O.swizzle_index(f, stages)] = logical[f]
    for kind in ("sum", "max", "argmax"):
        got = O.reduce(kind, physical, 0, [(N, M)], [(M, 1)], swizzle=stages)
        want = red[f"a_{kind}"]
        if kind == "sum":
            np.testing.assert_array_equal(got, want)
        else:
            np.testing.assert_array_equal(bits(got), bits(want))


def test_matmul_matches_reference_bit_for_bit():
    g = np.load(GOLDEN / "matmul.npz")
    np.testing.assert_array_equal(bits(O.matmul(g["lhs"], g["rhs"])), bits(g["out"]))
    np.testing.assert_array_equal(bits(O.matmul(g["lhs"], g["rhs"], acc64=True)), bits(g["out_acc64"]))
    assert "Stride<(1, 24)>" in str(g["out_layout"])  # canonical column-major result


def test_empty_fibre_is_rejected_for_extrema():
    x = np.zeros(4, dtype=np.float32)
    with pytest.raises(ValueError):
        O.reduce("max", x, 0, [(4, 1)], [(0, 1)])
    assert O.reduce("sum", x, 0, [(4, 1)], [(0, 1)]).tolist() == [0.0] * 4


# ---- MX element formats -------------------------------------------------------


def test_e4m3_codes_round_trip_exhaustively():
    for code in range(256):
        v = O.decode_elem(O.E4M3, code)
        if math.isnan(v):
            assert code & 0x7F == 0x7F
            continue
        assert O.encode_elem(O.E4M3, np.float32(v)) == code
    assert O.decode_elem(O.E4M3, 0x7E) == 448.0
    assert O.decode_elem(O.E4M3, 0x01) == 2.0 ** -9
    assert O.decode_elem(O.E4M3, 0x08) == 2.0 ** -6


def test_e2m1_codes_round_trip_exhaustively():
    values = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for code in range(16):
        v = O.decode_elem(O.E2M1, code)
        assert abs(v) == values[code & 7]
        assert O.encode_elem(O.E2M1, np.float32(v)) == code


@pytest.mark.parametrize(
    "value,code",
    [
        (464.0, 0x7E),   # tie between 448 (even) and the NaN slot: 448
        (470.0, 0x7E),   # rounds past the largest finite value: saturate
        (1e30, 0x7E),
        (-1e30, 0xFE),
        (2.0 ** -10, 0x00),  # half the smallest subnormal: ties to even (zero)
        (1.5 * 2.0 ** -10, 0x01),
        (7.5 * 2.0 ** -9, 0x08),  # subnormal rounding carries into the min normal
        (-0.0, 0x80),
        (1.0625, 0x38),  # 1 + 1/16 ties to even mantissa (1.0)
        (1.1875, 0x3A),  # 1 + 3/16 ties to even mantissa (1.25)
    ],
)
def test_e4m3_known_answers(value, code):
    assert O.encode_elem(O.E4M3, np.float32(value)) == code


@pytest.mark.parametrize(
    "value,code",
    [(0.25, 0x0), (0.75, 0x2), (1.25, 0x2), (1.75, 0x4), (2.5, 0x4), (3.5, 0x6), (5.0, 0x6), (7.0, 0x7),
     (1e9, 0x7), (-5.0, 0xE), (-0.0, 0x8)],
)
def test_e2m1_known_answers(value, code):
    assert O.encode_elem(O.E2M1, np.float32(value)) == code


def test_block_scale_rules():
    x = np.zeros((5, 32), dtype=np.float32)
    x[0, 3] = 1.0  # amax 1 -> e = -8 (E4M3)
    x[1, :] = -0.0  # zero block
    x[2, 4] = np.nan
    x[3, 5] = np.inf
    x[4, 0] = np.float32(2.0 ** -128)  # subnormal amax -> e clamped to -127
    x[4, 1] = np.float32(2.0 ** -140)  # far below the smallest element: zero
    p, s = O.mx_quantize(O.E4M3, x)
    assert s[:, 0].tolist() == [127 - 8, 0, 0xFF, 0xFF, 0]
    assert p[0, 3] == O.encode_elem(O.E4M3, np.float32(256.0))
    assert (p[1] == 0x80).all()  # zeros keep their sign
    assert (p[2] == 0).all() and (p[3] == 0).all()
    assert p[4, 0] == O.encode_elem(O.E4M3, np.float32(0.5)) and p[4, 1] == 0
    d = O.mx_dequantize(O.E4M3, p, s, 5, 32)
    assert d[0, 3] == 1.0 and np.isnan(d[2]).all() and np.isnan(d[3]).all()
    assert d[4, 0] == np.float32(2.0 ** -128) and d[4, 1] == 0.0  # exact binary32 subnormal
    p4, s4 = O.mx_quantize(O.E2M1, x)
    assert s4[0, 0] == 127 - 2 and (p4[0, 1] >> 4) == O.encode_elem(O.E2M1, np.float32(4.0))  # element 3: high nibble


def test_e4m3_payload_matches_torch_rounding_in_range():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((64, 256)) * np.exp(rng.uniform(-8, 8, size=(64, 1)))).astype(np.float32)
    p, s = O.mx_quantize(O.E4M3, x)
    scaled = x / np.repeat(np.ldexp(1.0, s.astype(np.int64) - 127), 32, axis=1)
    t = torch.from_numpy(scaled.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    in_range = np.abs(scaled) <= 448.0
    np.testing.assert_array_equal(t[in_range], p[in_range])
    assert (p[~in_range] & 0x7F == 0x7E).all()  # saturated, never NaN


def test_quantise_dequantise_error_bound():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((32, 128)).astype(np.float32)
    for fmt, mbits, emin, vmax in ((O.E4M3, 3, -6, 448.0), (O.E2M1, 1, 0, 6.0)):
        p, s = O.mx_quantize(fmt, x)
        d = O.mx_dequantize(fmt, p, s, 32, 128)
        scale = np.repeat(np.ldexp(1.0, s.astype(np.int64) - 127), 32, axis=1)
        q = np.abs(x.astype(np.float64)) / scale  # element units
        expo = np.maximum(np.floor(np.log2(np.maximum(q, 1e-300))), emin)
        spacing = np.ldexp(1.0, (expo - mbits).astype(np.int64))
        err = np.abs(d.astype(np.float64) - x) / scale
        saturated = q > vmax
        assert (err[~saturated] <= spacing[~saturated] / 2).all()
        assert (np.abs(d[saturated]) == (vmax * scale[saturated]).astype(np.float32)).all()


def test_tc128_scale_placement():
    # the 128 x 4 atom order consumed by tcgen05.cp .32x128b.warpx4
    assert O.scale_index_tc128(0, 0, 8) == 0
    assert O.scale_index_tc128(1, 0, 8) == 16
    assert O.scale_index_tc128(32, 0, 8) == 4
    assert O.scale_index_tc128(0, 3, 8) == 3
    assert O.scale_index_tc128(0, 4, 8) == 512
    assert O.scale_index_tc128(128, 0, 8) == 1024
    seen = {O.scale_index_tc128(r, kb, 8) for r in range(256) for kb in range(8)}
    assert len(seen) == 256 * 8 and max(seen) == O.scale_bytes_tc128(256, 8) - 1
    x = np.random.default_rng(2).standard_normal((256, 256)).astype(np.float32)
    p0, s0 = O.mx_quantize(O.E4M3, x)
    p1, s1 = O.mx_quantize(O.E4M3, x, scale_layout=1)
    np.testing.assert_array_equal(p0, p1)
    for r in range(0, 256, 37):
        for kb in range(8):
            assert s1[O.scale_index_tc128(r, kb, 8)] == s0[r, kb]
