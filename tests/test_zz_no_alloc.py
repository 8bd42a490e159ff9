"""The allocation-free attention backward (nl_flash_attention_bwd_noalloc).

Some callers cannot allocate device memory when they run the backward — for
example a host framework that hands the kernel only its own input and output
buffers, or code running where cudaMalloc is not allowed.  This entry point
takes no workspace: its scratch is a fixed array inside the library.  The test
calls it through the C ABI twice in a row (the shared scratch keeps the first
call's contents, so the second call checks that it is cleared) and compares
with the workspace-taking nl_flash_attention_bwd: dK and dV come from the same
kernels and accumulation order and must be bit-identical; dQ is summed by
reduce-adds whose order can vary, so it is held to the attention tests'
tolerance (max |err| / max |ref| <= 1e-2).  One case fills the array to its
last row, so a misplaced D vector would be caught there.  This file is collected last, and
also passes on its own in a fresh process."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200._lib import lib, ptr, stream_handle, check, STATUS  # noqa: E402
from nlearn_b200 import attention as A  # noqa: E402

TOL = 1e-2


def nrel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-3)).item()


def _noalloc(Q, K, V, O, dO, L):
    n, s, d = Q.shape
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(Q), torch.empty_like(Q)
    check(lib.nl_flash_attention_bwd_noalloc(ptr(Q), ptr(K), ptr(V), ptr(O), ptr(dO), ptr(L), ptr(dQ), ptr(dK),
                                             ptr(dV), n, s, d, stream_handle()), "nl_flash_attention_bwd_noalloc")
    return dQ, dK, dV


@pytest.mark.parametrize("n,s", [(32, 512), (6, 300), (256, 512)])
def test_noalloc_matches_workspace_entry(cuda, n, s):
    torch.manual_seed(n + s)
    Q, K, V, dO = (torch.randn(n, s, 64, device=cuda).bfloat16() for _ in range(4))
    O, L = A._flash_fwd_raw(Q, K, V)
    ref = A._flash_bwd_raw(Q, K, V, O, L, dO)       # nl_flash_attention_bwd, caller workspace
    for _ in range(2):                               # two calls in a row share the scratch
        got = _noalloc(Q, K, V, O, dO, L)
        torch.cuda.synchronize()
        assert nrel(got[0], ref[0]) < TOL
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])
    assert lib.nl_get_device_error(stream_handle()) == 0


def test_noalloc_rejects_oversize(cuda):
    cap = lib.nl_flash_attention_bwd_noalloc_max_rows()
    assert cap == 131072
    n, s = 2, cap // 2 + 128          # one head-row over the limit; nothing is launched
    st = lib.nl_flash_attention_bwd_noalloc(None, None, None, None, None, None, None, None, None, n, s, 64,
                                            stream_handle())
    assert STATUS[st] == "NL_ERR_TOO_LARGE"
