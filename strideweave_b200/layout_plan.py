"""Lowering of StrideWeave hierarchical layouts to the kernels' flat plans.

A ``Layout``'s top-level mode is a tree of (extent, stride) leaves.  The
kernels take each mode as a flat list of leaves in StrideWeave's
colexicographic order - first leaf fastest, exactly the order of
``LayoutCache::leaf_shapes`` / ``leaf_strides``
(src/strideweave/core/native/_layout_index.hpp:116-120) - plus the tensor
offset and, when the carrier stores its flat index space through a
``Swizzle``, the XOR stages of that swizzle
(src/strideweave/core/swizzle.py:107-117).
"""

from __future__ import annotations

from typing import Any

Leaf = tuple[int, int]


def _flatten(shape_level: Any, stride_level: Any, out: list[Leaf]) -> None:
    if isinstance(shape_level, int):
        out.append((int(shape_level), int(stride_level)))
        return
    for s, d in zip(shape_level, stride_level, strict=True):
        _flatten(s, d, out)


def mode_leaves(layout: Any, mode: int) -> list[Leaf]:
    """(extent, stride) leaves of top-level ``mode``, first leaf fastest."""
    leaves: list[Leaf] = []
    _flatten(layout.shape.top_level[mode], layout.stride.top_level[mode], leaves)
    return leaves


def all_leaves(layout: Any) -> list[Leaf]:
    leaves: list[Leaf] = []
    for mode in range(len(layout)):
        leaves.extend(mode_leaves(layout, mode))
    return leaves


def mode_size(layout: Any, mode: int) -> int:
    size = 1
    for extent, _ in mode_leaves(layout, mode):
        size *= extent
    return size


def coalesce(leaves: list[Leaf]) -> list[Leaf]:
    """Drop unit leaves and merge neighbours that walk memory contiguously in
    logical order; the result addresses the same elements in the same order."""
    out: list[Leaf] = []
    for extent, stride in leaves:
        if extent == 1:
            continue
        if out and out[-1][1] * out[-1][0] == stride:
            out[-1] = (out[-1][0] * extent, out[-1][1])
        else:
            out.append((extent, stride))
    return out


def single_stride(leaves: list[Leaf]) -> tuple[int, int] | None:
    """(extent, stride) when a mode walks memory with one stride, else None."""
    merged = coalesce(leaves)
    size = 1
    for extent, _ in leaves:
        size *= extent
    if not merged:
        return (size, 0)
    if len(merged) == 1:
        return merged[0]
    return None


def swizzle_stages(carrier: Any) -> list[tuple[int, int, int]]:
    swz = getattr(carrier, "swizzle", None)
    if swz is None:
        return []
    return [(int(s.bits), int(s.base), int(s.shift)) for s in swz.stages]


def swizzle_map(stages: list[tuple[int, int, int]], count: int) -> Any:
    """Physical index of flat indices 0 .. count-1 under the XOR stages, all at
    once: each stage r ^= ((r >> (base + shift)) & mask) << base, or for a
    negative shift r ^= ((r >> base) & mask) << (base - shift), in order -
    the map of src/strideweave/core/swizzle.py:107-117 over numpy arrays."""
    import numpy as np

    r = np.arange(count, dtype=np.int64)
    for bits, base, shift in stages:
        mask = (1 << bits) - 1
        if shift > 0:
            r ^= ((r >> (base + shift)) & mask) << base
        else:
            r ^= ((r >> base) & mask) << (base - shift)
    return r


def canonical_strides(shape_level: Any, stride: int = 1) -> tuple[Any, int]:
    """Column-major strides over a nested shape (the reference's canonical
    result layout, src/strideweave/carriers/cpu/native/_cpu_carrier.hpp:628-664)."""
    if isinstance(shape_level, int):
        return stride, stride * shape_level
    out = []
    nxt = stride
    for child in shape_level:
        s, nxt = canonical_strides(child, nxt)
        out.append(s)
    return out, nxt


def _as_python(shape_level: Any) -> Any:
    if isinstance(shape_level, int):
        return int(shape_level)
    return [_as_python(child) for child in shape_level]


def canonical_layout(*mode_shapes: Any) -> Any:
    """Canonical (first-mode-fastest, compact) layout over the given modes."""
    from ._host import Layout, Shape, Stride

    modes = [_as_python(m) for m in mode_shapes]
    shape = Shape(modes[0]) if len(modes) == 1 else Shape(modes)
    strides, _ = canonical_strides(shape.top_level, 1)
    return Layout(shape, Stride(strides))


def injective_layout_for(layout: Any) -> Any:
    """``layout`` when it is injective, else the canonical layout of its shape
    (where a gradient of that tensor is stored)."""
    if layout.is_injective:
        return layout
    return canonical_layout(*[layout.shape.top_level[m] for m in range(len(layout))])


def view_extent(offset: int, leaves: list[Leaf]) -> tuple[int, int]:
    """Smallest and largest flat index a view touches (before any swizzle)."""
    lo = hi = offset
    for extent, stride in leaves:
        if extent <= 0:
            return offset, offset - 1
        span = (extent - 1) * stride
        if span < 0:
            lo += span
        else:
            hi += span
    return lo, hi
