"""fhe_rescale_noalloc: the rescale for callers that cannot let the library
allocate device memory (a framework that owns every allocation, or a memory
budget fixed in advance).  Its scratch is a fixed device array inside the
library, so the caller passes only its own input and output buffers.

The test calls it through the C ABI twice in a row on different ciphertexts
and checks each result word for word against the ordinary fhe_rescale entry
point (rescale is exact integer work, so the tolerance is equality).  It also
checks that a size above the fixed maximum is rejected.  This file is named to
be collected last; it passes alone in a fresh process and after the others.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rand_ct(q, nq, n, seed):
    rng = np.random.default_rng(seed)
    x = np.empty((2, nq, n), dtype=np.uint64)
    for l in range(nq):
        x[:, l, :] = rng.integers(0, q[l], size=(2, n), dtype=np.uint64)
    return x


def _noalloc(cc, x):
    import torch
    from fhe_mamba_b200 import _lib
    d_in = torch.from_numpy(x.view(np.int64).copy()).cuda()
    d_out = torch.empty((x.shape[0], x.shape[1] - 1, x.shape[2]), dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    _lib.call("fhe_rescale_noalloc", cc.h, ctypes.c_void_p(d_in.data_ptr()), x.shape[0], x.shape[1],
              ctypes.c_void_p(d_out.data_ptr()))
    cc.synchronize()
    return d_out.cpu().numpy().view(np.uint64)


def test_noalloc_rescale_matches_fhe_rescale_twice():
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 14, multiplicative_depth=8, scaling_mod_size=50,
                                first_mod_size=60, num_large_digits=2))
    for call, nq in enumerate((cc.n_q, 5)):
        x = _rand_ct(cc.q, nq, cc.n, 100 + call)
        ref = cc.upload(x)
        cc.RescaleInPlace(ref)
        want = ref.residues()
        got = _noalloc(cc, x)
        assert np.array_equal(got, want), f"call {call}"


@pytest.mark.parametrize("ncomp", [1, 3])
def test_noalloc_rescale_one_and_three_components(ncomp):
    """A single residue polynomial (compared with component 0 of a two-component
    rescale: rescaling works on each component alone) and a 3-component
    product before relinearisation."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 14, multiplicative_depth=8, scaling_mod_size=50,
                                first_mod_size=60, num_large_digits=2))
    x = _rand_ct(cc.q, cc.n_q, cc.n, 200 + ncomp)
    if ncomp == 3:
        x = np.concatenate([x, _rand_ct(cc.q, cc.n_q, cc.n, 300)[:1]])
    ref = cc.upload(x, noise_deg=2 if ncomp == 3 else 1)
    cc.RescaleInPlace(ref)
    want = ref.residues()[:ncomp]
    for _ in range(2):
        assert np.array_equal(_noalloc(cc, x[:ncomp]), want)


def test_noalloc_rejects_overlapping_output():
    import torch
    from fhe_mamba_b200 import CCParams, CryptoContext, InvalidArgument, _lib
    cc = CryptoContext(CCParams(ring_dim=1 << 14, multiplicative_depth=8, scaling_mod_size=50,
                                first_mod_size=60, num_large_digits=2))
    buf = torch.zeros(2 * cc.n_q * cc.n, dtype=torch.int64, device="cuda")
    shifted = ctypes.c_void_p(buf.data_ptr() + cc.n * 8)
    with pytest.raises(InvalidArgument, match="overlap"):
        _lib.call("fhe_rescale_noalloc", cc.h, ctypes.c_void_p(buf.data_ptr()), 2, cc.n_q, shifted)


def test_noalloc_rejects_sizes_above_its_fixed_scratch():
    import torch
    from fhe_mamba_b200 import CCParams, CryptoContext, InvalidArgument, _lib
    cc = CryptoContext(CCParams(ring_dim=1 << 17, multiplicative_depth=39, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=4))
    small = torch.zeros(16, dtype=torch.int64, device="cuda")
    with pytest.raises(InvalidArgument, match="maximum"):
        _lib.call("fhe_rescale_noalloc", cc.h, ctypes.c_void_p(small.data_ptr()), 2, 40,
                  ctypes.c_void_p(small.data_ptr()))
