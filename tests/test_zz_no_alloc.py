"""GPU check of ``bsa_sampled_mass_noalloc`` (the entry point that allocates
nothing) against the workspace path ``bsa_sampled_mass``, through the C ABI.

The file name sorts last so the suite runs it after every other GPU test; it
also passes on its own in a fresh process.
"""

import math

import pytest
import torch

from dit_sparse_atten_b200 import _native, kernels

pytestmark = pytest.mark.gpu

DEV = "cuda"
SCRATCH_BYTES = 32 << 20   # the library's static scratch (bsa_kernels.h)
ATOL = 1e-6                # mass cells are probabilities in [0, 1]
RTOL = 1e-5


def noalloc_mass(q, k, block, samples, scale=None, round_bf16=True):
    B, T, H, D = q.shape
    blocks = math.ceil(T / block)
    mass = torch.empty((B, H, blocks, blocks), dtype=torch.float32, device=q.device)
    s = float(scale) if scale is not None else D ** -0.5
    _native.call("bsa_sampled_mass_noalloc", q.data_ptr(), k.data_ptr(), B, T, H, D, block,
                 samples, s, 1 if round_bf16 else 0, mass.data_ptr(),
                 _native.err_word(q.device).data_ptr(),
                 torch.cuda.current_stream(q.device).cuda_stream)
    return mass


def inputs(B, T, H, seed):
    g = torch.Generator().manual_seed(seed)
    q, k = (torch.randn((B, T, H, 128), generator=g).to(torch.bfloat16).to(DEV)
            for _ in range(2))
    return q, k


@pytest.mark.parametrize("B,T,H,block,samples", [
    (1, 4096, 3, 128, 2),       # whole blocks, the reference's default S
    (2, 3000, 5, 128, 16),      # partial last block (56 tokens), S of config 3
    (1, 57600, 12, 128, 16),    # config-3 rows: 7,200 sampled rows, several head chunks
])
def test_matches_workspace_path_twice(B, T, H, block, samples):
    q, k = inputs(B, T, H, seed=T + H)
    ref = kernels.sampled_block_mass(q, k, block, samples, one_pass=False)
    for _ in range(2):
        got = noalloc_mass(q, k, block, samples)
        torch.cuda.synchronize()
        _native.check_device_errors()
        torch.testing.assert_close(got, ref, atol=ATOL, rtol=RTOL)


def test_allocates_nothing_and_rewrites_its_scratch():
    """After a warm-up call, a call changes neither torch's allocated bytes nor
    the device's free memory; a large case followed by a smaller one with other
    inputs still matches the workspace path, so every call writes all of the
    scratch it reads (nothing is left over from the call before)."""
    big_q, big_k = inputs(1, 57600, 12, seed=11)
    small_q, small_k = inputs(2, 3000, 5, seed=12)
    small_ref = kernels.sampled_block_mass(small_q, small_k, 128, 16, one_pass=False)
    big_mass = torch.empty((1, 12, 450, 450), dtype=torch.float32, device=DEV)
    small_mass = torch.empty_like(small_ref)

    def call(q, k, out):
        _native.call("bsa_sampled_mass_noalloc", q.data_ptr(), k.data_ptr(), q.shape[0],
                     q.shape[1], q.shape[2], 128, 128, 16, 128 ** -0.5, 1, out.data_ptr(),
                     _native.err_word(q.device).data_ptr(),
                     torch.cuda.current_stream(q.device).cuda_stream)

    call(big_q, big_k, big_mass)               # warm-up: set-up happens here
    torch.cuda.synchronize()
    allocated, free = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    call(big_q, big_k, big_mass)
    call(small_q, small_k, small_mass)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.cuda.memory_allocated() == allocated
    assert torch.cuda.mem_get_info()[0] == free
    torch.testing.assert_close(small_mass, small_ref, atol=ATOL, rtol=RTOL)


def test_rejects_sizes_beyond_the_scratch():
    # 2049 blocks x 32 samples = 65,568 sampled rows: 2 * 65,568 * 256 bytes for
    # one head already exceeds the 32 MiB scratch.  The call must fail before
    # launching anything.
    T = 2049 * 128
    assert 2 * 2049 * 32 * 256 > SCRATCH_BYTES
    q = torch.zeros((1, T, 1, 128), dtype=torch.bfloat16, device=DEV)
    mass = torch.empty((1, 1, 2049, 2049), dtype=torch.float32, device=DEV)
    rc = _native.load_library().bsa_sampled_mass_noalloc(
        q.data_ptr(), q.data_ptr(), 1, T, 1, 128, 128, 32, 128 ** -0.5, 1, mass.data_ptr(),
        _native.err_word(q.device).data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"scratch" in _native.load_library().bsa_last_error()
