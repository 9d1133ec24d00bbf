"""The kernels' bounded mbarrier wait, made to run out on purpose.

A diagnostic kernel (test-only ``libbsa_diag.so``) waits with the product's
``mbar_wait_for`` on an mbarrier that nothing arrives on, with a 1 ms limit.
The wait must return, report ``kErrWaitTimeout`` in the caller's error word
and raise the CTA's abort flag; the host must turn the word into a
``RuntimeError``; and the next normal launches on the device must succeed
(the context stays usable).  No trap, no fault, no unbounded wait.
"""

import pytest
import torch

from dit_sparse_atten_b200 import _native, kernels

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000          # 1 ms


def test_unarmed_wait_times_out_and_reports():
    import diag

    device = torch.device("cuda", torch.cuda.current_device())
    word = _native.err_word(device)
    _native.check_device_errors()                     # start from a clear word
    completed, elapsed_ns, abort = diag.unarmed_wait(LIMIT_NS, word)
    assert completed == 0
    assert abort == 1
    assert LIMIT_NS <= elapsed_ns < 500 * LIMIT_NS
    assert int(word.item()) & 1                        # BSA_DEVICE_WAIT_TIMEOUT
    with pytest.raises(RuntimeError, match="timed out"):
        _native.check_device_errors()
    assert int(word.item()) == 0                       # cleared by the check


def test_device_usable_after_timeout():
    import diag

    device = torch.device("cuda", torch.cuda.current_device())
    word = _native.err_word(device)
    diag.unarmed_wait(LIMIT_NS, word)
    with pytest.raises(RuntimeError):
        _native.check_device_errors()
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn((1, 384, 2, 128), generator=g).to(torch.bfloat16).to(device)
               for _ in range(3))
    perm = torch.randperm(384, generator=g).to(torch.int32).to(device)
    (qp,) = kernels.reorder_rows([q], perm)
    route = torch.ones((2, 3, 3), dtype=torch.bool, device=device)
    counts, indices = kernels.pack_boolean_rows(route)
    out = kernels.block_sparse_attention(q, k, v, counts, indices, block=128)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(qp, q[:, perm.long()])
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2).float(), k.transpose(1, 2).float(), v.transpose(1, 2).float())
    assert (out.float() - ref.transpose(1, 2)).abs().max() < 2e-2
