"""The bounds-checked build (`python build_ext.py --debug` -> `_Cdbg`): an out-of-range index is recorded, the access
is skipped and the context stays usable - the stand-in for a memory checker on machines where none may run."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dbg():
    try:
        return importlib.import_module("modded_nanogpt_b200._Cdbg")
    except ImportError:
        pytest.skip("debug extension not built (python build_ext.py --debug)")


def test_out_of_range_embedding_rows_are_recorded_not_written():
    C = _dbg()
    assert C.bounds_checked_build()
    V, D, n = 1000, 768, 4096
    g = torch.randn(n, D, device="cuda").bfloat16()
    ids = torch.randint(0, V, (n,), device="cuda")
    grad = torch.zeros(V, D, dtype=torch.bfloat16, device="cuda")
    sorted_ids, perm = torch.sort(ids)
    C.embed_bwd(g, sorted_ids, perm, grad)
    assert C.bounds_status() == 0
    want = torch.zeros(V, D, device="cuda").index_add_(0, ids, g.float())
    assert ((grad.float() - want).norm() / want.norm()).item() < 1e-2
    # the same call with ids beyond the table: nothing outside `grad` is touched (canary rows), the bad rows are dropped
    bad = ids.clone()
    bad[::7] = V + 5
    bad[3] = -2
    buf = torch.full((V + 16, D), 3.0, dtype=torch.bfloat16, device="cuda")
    grad2 = buf[8:8 + V]
    grad2.zero_()
    sorted_ids, perm = torch.sort(bad)
    C.embed_bwd(g, sorted_ids, perm, grad2)
    line = C.bounds_status()
    assert line > 0                                          # the source line of the check that fired
    assert C.bounds_status() == 0                            # reading clears the word
    assert (buf[:8] == 3.0).all() and (buf[8 + V:] == 3.0).all()
    keep = (bad >= 0) & (bad < V)
    want2 = torch.zeros(V, D, device="cuda").index_add_(0, bad[keep], g.float()[keep])
    assert ((grad2.float() - want2).norm() / want2.norm()).item() < 1e-2
    torch.cuda.synchronize()                                 # the context is alive


def test_regular_build_has_no_checks():
    from modded_nanogpt_b200.ops import native
    assert not native.lib().bounds_checked_build() and native.lib().bounds_status() == 0
