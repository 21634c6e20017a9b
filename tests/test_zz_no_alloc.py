"""The allocation-free entry point `mng_quant_transpose_e4m3_static`, called through its exported
C symbol the way a host program without an allocator at hand would call it (it brings its own
input and output buffers, the library brings the scratch).  Its output must equal the regular
entry point's, also on a second call that reuses the built-in scratch array with other data and
a different width.  Collected last so that a stop-at-first-failure run has already covered every
other test; passes alone in a fresh process as well."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _load():
    from modded_nanogpt_b200.ops import native
    mod = native.lib()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.mng_quant_transpose_e4m3_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_void_p]
    lib.mng_static_strerror.restype = ctypes.c_char_p
    lib.mng_static_strerror.argtypes = [ctypes.c_int]
    return mod, lib, fn


def test_static_scratch_entry_point_matches_regular_one():
    mod, lib, fn = _load()
    torch.manual_seed(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream().cuda_stream
    for call, (rows, cols, scale_in) in enumerate([(768, 3072, 0.02), (1000, 300, 3.0)]):
        src = (torch.randn(rows, cols, device=dev) * scale_in).to(torch.bfloat16)
        want_q = torch.empty(cols, rows, dtype=torch.float8_e4m3fn, device=dev)
        want_s = torch.empty(cols, dtype=torch.float32, device=dev)
        mod.quant_transpose(src, want_q, want_s, torch.empty(cols, dtype=torch.int32, device=dev))
        got_q = torch.zeros(cols, rows, dtype=torch.float8_e4m3fn, device=dev)
        got_s = torch.zeros(cols, dtype=torch.float32, device=dev)
        rc = fn(src.data_ptr(), got_q.data_ptr(), got_s.data_ptr(), rows, cols, stream)
        assert rc == 0, lib.mng_static_strerror(rc)
        torch.cuda.synchronize()
        assert torch.equal(got_s, want_s), f"scales differ on call {call}"
        assert torch.equal(got_q.view(torch.uint8), want_q.view(torch.uint8)), f"payload differs on call {call}"
        # and both agree with the plain fp32 statement of the op
        ref_s = src.float().abs().amax(0) / 448
        assert torch.allclose(got_s, ref_s, rtol=1e-6)
        deq = got_q.float() * got_s[:, None]
        assert ((deq - src.float().T).norm() / src.float().norm()).item() < 4e-2


def test_static_scratch_entry_point_rejects_oversize():
    _, lib, fn = _load()
    x = torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), 8, 65537, torch.cuda.current_stream().cuda_stream)
    assert rc == -22 and b"65536" in lib.mng_static_strerror(rc)
    assert fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 8, None) == -24
    # more rows than the kernels' launch grid covers: refused up front, not reported as a failed launch
    assert fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), 65535 * 64 + 1, 8, torch.cuda.current_stream().cuda_stream) == -22
