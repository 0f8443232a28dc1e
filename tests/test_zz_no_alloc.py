"""chm_forward_noalloc: the forward for callers that cannot allocate device
memory (a plugin host that lends only its own input/output buffers, a
foreign-language binding without a device allocator, code that must not
trigger cudaMalloc's device synchronisation). Its scratch is a static
device array inside the library, so the caller passes only inputs and
outputs.

Checked through the C ABI against the regular workspace-based forward
(chm_forward via the model) on two calls in a row: the same kernels run on
the same inputs, so the outputs must be bitwise equal (a scratch-layout or
aliasing fault would show up as any difference at all). The status word
kept in the static scratch (chm_noalloc_read_status) reads back clean
after the calls, and a batch whose scratch would not fit is rejected.
This file is collected last on purpose.
"""

import ctypes

import pytest
import torch

import cherimoya_b200 as cb
from cherimoya_b200 import _lib, ops
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

CHM_ERR_WORKSPACE = 3


def _noalloc(lib, desc, packed_ptr, X, profile, logcounts):
    return lib.chm_forward_noalloc(
        ctypes.byref(desc), ctypes.c_void_p(packed_ptr), X.shape[0], ctypes.c_void_p(X.data_ptr()),
        _lib.INPUT_F32, None, ctypes.c_void_p(profile.data_ptr()),
        ctypes.c_void_p(logcounts.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_noalloc_forward_matches_workspace_forward(mode):
    lib = _lib.load()
    torch.manual_seed(0)
    model = cb.Cherimoya(compile=False, precision=mode).eval().to("cuda")
    g = torch.Generator().manual_seed(3)
    X = O.one_hot(torch.randint(0, 4, (8, 2114), generator=g)).to("cuda")
    with torch.no_grad():
        ref_p, ref_c = model(X)
    buf, off = model.engine_weights(X.device)
    mode_id = _lib.MODE_FP32 if mode == "fp32" else _lib.MODE_BF16
    desc = ops._desc(model.engine_desc(X.shape[-1], mode_id), float(model.residual_scale))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):   # two calls in a row share the static scratch
        prof = torch.full_like(ref_p, float("nan"))
        lc = torch.full_like(ref_c, float("nan"))
        assert _noalloc(lib, desc, buf.data_ptr() + off, X, prof, lc) == 0
        assert lib.chm_noalloc_read_status(stream) == 0
        assert torch.equal(prof, ref_p) and torch.equal(lc, ref_c)


def test_noalloc_rejects_batch_beyond_static_scratch():
    lib = _lib.load()
    torch.manual_seed(0)
    model = cb.Cherimoya(compile=False).eval().to("cuda")
    buf, off = model.engine_weights(torch.device("cuda"))
    desc = ops._desc(model.engine_desc(2114, _lib.MODE_FP32), float(model.residual_scale))
    small = torch.zeros(1, 4, 2114, device="cuda")
    prof = torch.zeros(1, 1, 1000, device="cuda")
    lc = torch.zeros(1, 1, device="cuda")
    # 64 fp32 sequences of 2114 bp need ~138 MB of scratch: rejected before any launch
    st = lib.chm_forward_noalloc(
        ctypes.byref(desc), ctypes.c_void_p(buf.data_ptr() + off), 64,
        ctypes.c_void_p(small.data_ptr()), _lib.INPUT_F32, None,
        ctypes.c_void_p(prof.data_ptr()), ctypes.c_void_p(lc.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == CHM_ERR_WORKSPACE
