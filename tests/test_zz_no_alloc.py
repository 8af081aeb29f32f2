"""The allocation-free total order (pxb_total_order_noalloc) against the
scratch-taking pxb_total_order, through the C ABI.

Callers that cannot allocate device memory (an FFI handler under CUDA-graph
capture, a plugin whose host owns all device memory) use this entry point;
its scratch is a fixed array inside libpxb.so. Two calls in a row must both
give exactly the permutation of pxb_total_order (the second call finds the
first call's leftovers in the shared array), and a size past the array's
limit is refused with an error instead of running.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_N = 1 << 18


def _inputs(rng, m, id_bound):
    score = (np.floor(rng.random(m) * 64) / 8).astype(np.float32)  # many ties
    score[rng.integers(0, m, m // 20)] = -np.inf
    score[rng.integers(0, m, m // 50)] = np.nan
    src = rng.integers(0, min(id_bound, 300), m).astype(np.int32)
    dst = rng.integers(0, id_bound, m).astype(np.int32)
    return score, src, dst


def _noalloc(score_d, src_d, dst_d, id_bound, out):
    import torch

    from plastax_b200 import _lib
    from plastax_b200.kernels import _stream, ptr

    _lib.call("pxb_total_order_noalloc", ctypes.c_int64(score_d.numel()), ptr(score_d), ptr(src_d), ptr(dst_d),
              ctypes.c_int32(id_bound), ptr(out), _stream())
    torch.cuda.synchronize()
    return out.cpu().numpy().copy()


@pytest.mark.parametrize("m,id_bound", [(MAX_N, 1_048_592), (100_000, 65_536), (3_000, 50)])
def test_noalloc_total_order_matches_scratch_version_twice(cuda, m, id_bound):
    import torch

    from plastax_b200 import kernels

    rng = np.random.default_rng(m)
    outs = []
    for call in range(2):
        score, src, dst = _inputs(rng, m, id_bound)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        s_d, a_d, b_d = t(score), t(src), t(dst)
        ref = kernels.total_order(s_d, a_d, b_d, id_bound).cpu().numpy()
        got = _noalloc(s_d, a_d, b_d, id_bound, torch.empty(m, dtype=torch.int32, device=cuda))
        np.testing.assert_array_equal(got, ref, err_msg=f"call {call}")
        outs.append(got)
    assert outs[0].shape == outs[1].shape


def test_noalloc_smaller_call_after_a_larger_one(cuda):
    """Calls of different sizes and id bounds in a row: a small call after
    the largest one (the array then holds the larger call's keys and CUB
    state past the new n), then the largest again, each equal to the
    scratch-taking version."""
    import torch

    from plastax_b200 import kernels

    rng = np.random.default_rng(7)
    for m, id_bound in [(MAX_N, 1_048_592), (3_000, 50), (100_000, 65_536), (MAX_N, 1_048_592), (17, 3)]:
        score, src, dst = _inputs(rng, m, id_bound)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        s_d, a_d, b_d = t(score), t(src), t(dst)
        ref = kernels.total_order(s_d, a_d, b_d, id_bound).cpu().numpy()
        got = _noalloc(s_d, a_d, b_d, id_bound, torch.empty(m, dtype=torch.int32, device=cuda))
        np.testing.assert_array_equal(got, ref, err_msg=f"m={m} id_bound={id_bound}")


def test_noalloc_rejects_more_than_its_array_holds(cuda):
    import torch

    from plastax_b200._lib import PxbError

    m = MAX_N + 1
    rng = np.random.default_rng(1)
    score, src, dst = _inputs(rng, m, 1000)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    with pytest.raises(PxbError, match="exceeds the maximum"):
        _noalloc(t(score), t(src), t(dst), 1000, torch.empty(m, dtype=torch.int32, device=cuda))
