"""Data movement as index maps: slice, transpose, reshape and concat fused
into the elementwise kernels that consume them.

The reference gives each movement op its own kernel and launch: ``slice``
(kernel_generator.py:1112-1240), ``transpose`` (:1949-1972), ``reshape``
(:2067-2086, a copy) and ``concat`` along axis 0 (:2092-2132).  None of them
computes anything, so here each is a *view*: a map from the coordinates of
its output to a flat offset in a tensor that exists in memory.  An
elementwise kernel reading the view reads that tensor through the map, and
the view itself is never written -- ``relu(transpose(slice(x)))`` is one
kernel that reads ``x`` once and writes the result once.

A map is a nested tuple over the output coordinates ``k``:

* ``("aff", src, base, strides)`` -- offset ``base + sum(k[i] * strides[i])``
  into tensor ``src``;
* ``("pw", axis, thr, lo, hi)`` -- map ``lo`` where ``k[axis] < thr``, else
  ``hi`` (a concat).

Views compose: a slice or transpose of a view is a view of the same tensors
(coordinate permutation plus offset); a reshape composes only with a view
that is the whole tensor in row-major order.  A view that cannot stay one --
fetched, read by a library kernel, read through a broadcast, read in another
phase, or whose source is overwritten before its last reader -- is written to
memory where it is defined (``steps.resolve_views``).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

Map = tuple


def rowmajor(shape: Sequence[int]) -> Tuple[int, ...]:
    out, acc = [], 1
    for d in reversed(tuple(int(x) for x in shape)):
        out.append(acc)
        acc *= d
    return tuple(reversed(out))


def identity(shape: Sequence[int], src: str) -> Map:
    return ("aff", src, 0, rowmajor(shape))


def leaves(m: Map) -> List[str]:
    if m[0] == "aff":
        return [m[1]]
    return leaves(m[3]) + [s for s in leaves(m[4]) if s not in leaves(m[3])]


def transform(m: Map, perm: Sequence[int], off: Sequence[int], out_shape: Sequence[int]) -> Map:
    """The map over coordinates ``k'`` (shape ``out_shape``) of a view whose
    input coordinates are ``in[a] = k'[perm[a]] + off[a]``, given the input's
    map ``m``."""
    out_shape = tuple(int(d) for d in out_shape)
    if m[0] == "aff":
        _, src, base, s = m
        strides = [0] * len(out_shape)
        for a, sa in enumerate(s):
            base += sa * int(off[a])
            strides[perm[a]] += sa
        return ("aff", src, int(base), tuple(int(x) for x in strides))
    _, axis, thr, lo, hi = m
    nax = perm[axis]
    nthr = int(thr) - int(off[axis])
    if nthr <= 0:
        return transform(hi, perm, off, out_shape)
    if nthr >= out_shape[nax]:
        return transform(lo, perm, off, out_shape)
    return ("pw", nax, nthr, transform(lo, perm, off, out_shape), transform(hi, perm, off, out_shape))


def is_whole(m: Map, shape: Sequence[int]) -> bool:
    """``m`` reads a whole tensor in row-major order (a reshape may follow)."""
    return m[0] == "aff" and m[2] == 0 and tuple(m[3]) == rowmajor(shape)


def rename(m: Map, f) -> Map:
    """The same map with each source name replaced by ``f(name)``."""
    if m[0] == "aff":
        return ("aff", f(m[1]), m[2], m[3])
    return ("pw", m[1], m[2], rename(m[3], f), rename(m[4], f))


def vec4_ok(m: Map, ndim: int) -> bool:
    """Four consecutive elements along the last axis are four consecutive,
    16-byte aligned floats of one source."""
    if m[0] == "aff":
        s = m[3]
        return (ndim > 0 and s[-1] == 1 and m[2] % 4 == 0
                and all(x % 4 == 0 for x in s[:-1]))
    return (m[1] != ndim - 1 or m[2] % 4 == 0) and vec4_ok(m[3], ndim) and vec4_ok(m[4], ndim)


class View:
    """A movement op as a map builder: ``build(maps, shapes)`` returns the
    output's map from the maps of its inputs, or None when the op cannot be
    expressed as a map of them (a reshape of a strided view)."""

    def __init__(self, kind: str, out: str, out_shape, sources: Sequence[str], params: tuple):
        self.kind, self.out = kind, out
        self.out_shape = tuple(int(d) for d in out_shape)
        self.sources = list(sources)
        self.params = params

    def build(self, in_maps: Sequence[Map], in_shapes) -> Optional[Map]:
        k, shp = self.kind, self.out_shape
        if k == "transpose":
            return transform(in_maps[0], (1, 0), (0, 0), shp)
        if k == "slice":
            return transform(in_maps[0], tuple(range(len(shp))), self.params, shp)
        if k == "reshape":
            m = in_maps[0]
            if not is_whole(m, in_shapes[0]):
                return None
            return ("aff", m[1], 0, rowmajor(shp))
        if k == "concat0":
            r1 = int(in_shapes[0][0])
            lo = transform(in_maps[0], tuple(range(len(shp))), (0,) * len(shp), shp)
            hi = transform(in_maps[1], tuple(range(len(shp))), (-r1,) + (0,) * (len(shp) - 1), shp)
            if r1 <= 0:
                return hi
            if r1 >= shp[0]:
                return lo
            return ("pw", 0, r1, lo, hi)
        raise ValueError(k)
