"""GPU test of j4b_reduce_sum_noalloc, the full sum for callers that cannot allocate device
memory while they run (a host with a fixed device-memory budget, a serving loop that must not
enter the allocator). It must give the same sum as the allocating j4b_reduce_sum, call after
call, although its scratch is one static device array that every call reuses. Collected last
so a failure here never hides the rest."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT = 134_217_728  # elements: 65,536 partials of 2,048 in the static scratch


def _noalloc(ptr, n, out):
    from jax4j_b200 import _lib
    from jax4j_b200.backend import torch_stream
    _lib.call("j4b_reduce_sum_noalloc", ptr, n, out.data_ptr(), torch_stream())


def test_noalloc_sum_matches_allocating_sum_twice_in_a_row(backend):
    rng = np.random.default_rng(42)
    # two calls in a row with different sizes: the second must not see the first's partials or
    # its arrival counter
    for n in (3_000_017, 4_099):
        a = rng.standard_normal(n).astype(np.float32)
        buf = backend.upload(a, (n,))
        want = backend.download(backend.reduce_sum(buf))[0]
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(buf.ptr, n, out)
        got = float(out.cpu()[0])
        # same bar as the dense reduction tests: the sums differ only in their rounding
        assert abs(got - float(want)) <= 1e-6 * max(1.0, float(np.abs(a).sum())), (n, got, want)


def test_noalloc_sum_at_its_size_limit(backend):
    """Exactly 134,217,728 elements (every partial slot of the scratch), twice in a row."""
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(LIMIT, device="cuda", generator=g)
    buf = backend.wrap(a)
    want = float(backend.download(backend.reduce_sum(buf))[0])
    bound = 1e-6 * float(a.abs().sum().item())
    for _ in range(2):
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(a.data_ptr(), LIMIT, out)
        got = float(out.cpu()[0])
        assert abs(got - want) <= bound, (got, want)


def test_noalloc_sum_rejects_bad_arguments(backend):
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="at most 134217728 elements"):
        _noalloc(out.data_ptr(), LIMIT + 1, out)
    host = torch.ones(16, dtype=torch.float32).pin_memory()  # not device memory: refused before any launch
    with pytest.raises(ValueError, match="not device memory"):
        _noalloc(host.data_ptr(), 16, out)
