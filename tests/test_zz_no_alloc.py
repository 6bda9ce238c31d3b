"""GPU test of j4b_reduce_sum_noalloc, the full sum for callers that cannot allocate device
memory while they run (stream capture in global mode, fixed memory budgets). It must give the
same sum as the allocating j4b_reduce_sum, call after call, although its scratch is one static
device array that every call reuses. Collected last so a failure here never hides the rest."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_noalloc_sum_matches_allocating_sum_twice_in_a_row(backend):
    from jax4j_b200 import _lib
    from jax4j_b200.backend import torch_stream
    rng = np.random.default_rng(42)
    # two calls in a row with different sizes: the second must not see the first's partials or
    # its arrival counter
    for n in (3_000_017, 4_099):
        a = rng.standard_normal(n).astype(np.float32)
        buf = backend.upload(a, (n,))
        want = backend.download(backend.reduce_sum(buf))[0]
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        _lib.call("j4b_reduce_sum_noalloc", buf.ptr, n, out.data_ptr(), torch_stream())
        got = float(out.cpu()[0])
        # same bar as the dense reduction tests: the sums differ only in their rounding
        assert abs(got - float(want)) <= 1e-6 * max(1.0, float(np.abs(a).sum())), (n, got, want)


def test_noalloc_sum_rejects_sizes_beyond_its_scratch(backend):
    from jax4j_b200 import _lib
    from jax4j_b200.backend import torch_stream
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="at most 134217728 elements"):
        _lib.call("j4b_reduce_sum_noalloc", out.data_ptr(), 134_217_729, out.data_ptr(),
                  torch_stream())
