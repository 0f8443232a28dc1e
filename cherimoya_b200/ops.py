"""torch custom ops over the C ABI (``cherimoya_b200::*``).

Each op allocates its outputs and its workspace from torch's caching
allocator on the current stream and calls into libcherimoya_b200.so; the
library itself never allocates, never synchronises, and never falls back
to another implementation. Fake (meta) implementations are registered so
``torch.compile`` can trace models that call these ops.
"""

import ctypes
from typing import List, Optional, Tuple

import torch

from . import _lib

ALIGN = 1024

# desc list layout shared by every op:
# [n_filters, n_layers, expansion, n_outputs, n_groups, n_control_tracks,
#  trimming, seq_len, mode]
D_C, D_NL, D_EXP, D_NOUT, D_NG, D_NCTL, D_T, D_L, D_MODE = range(9)


def _desc(desc, residual_scale):
    return _lib.make_desc(desc[D_C], desc[D_NL], desc[D_EXP], desc[D_NOUT], desc[D_NG],
                          desc[D_NCTL], desc[D_T], desc[D_L], residual_scale, desc[D_MODE])


def aligned_empty(nbytes, device):
    """uint8 device buffer with a 1024-byte-aligned window of `nbytes`;
    returns (tensor, byte offset of the window)."""
    buf = torch.empty(int(nbytes) + ALIGN, dtype=torch.uint8, device=device)
    return buf, (-buf.data_ptr()) % ALIGN


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(t, name):
    if not t.is_cuda:
        raise RuntimeError("cherimoya_b200: {} must be a CUDA tensor".format(name))


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


# ----------------------------------------------------------------- packing
def pack_weights(params, desc, residual_scale, device):
    """Pack fp32 parameters (dict of CUDA tensors in state_dict names,
    per-layer entries as lists) into the kernel layout. Returns
    (buffer, offset)."""
    lib = _lib.load()
    d = _desc(desc, residual_scale)
    _lib.check(lib.chm_validate(ctypes.byref(d)), "pack_weights")
    nbytes = lib.chm_packed_weights_bytes(ctypes.byref(d))
    buf, off = aligned_empty(nbytes, device)
    keep = []

    def f32(t):
        t = t.detach().to(device=device, dtype=torch.float32).contiguous()
        keep.append(t)
        return t.data_ptr()

    n_layers = desc[D_NL]
    arr = ctypes.c_void_p * max(n_layers, 1)
    cw = arr(*[f32(t) for t in params["conv_weight"]])
    w1 = arr(*[f32(t) for t in params["linear1_weight"]])
    w2 = arr(*[f32(t) for t in params["linear2_weight"]])
    p = _lib.Params(f32(params["iconv_weight"]), f32(params["iconv_bias"]), cw, w1, w2,
                    f32(params["fconv_weight"]), f32(params["fconv_bias"]),
                    f32(params["linear_weight"]), f32(params["linear_bias"]))
    st = lib.chm_pack_weights(ctypes.byref(d), ctypes.byref(p),
                              ctypes.c_void_p(buf.data_ptr() + off), nbytes, _stream(device))
    _lib.check(st, "pack_weights")
    # the fp32 temporaries must outlive the asynchronous pack kernels
    torch.cuda.current_stream(device).synchronize()
    return buf, off


# ----------------------------------------------------------------- forward
def _out_shapes(desc, N):
    Lout = desc[D_L] - 2 * desc[D_T]
    return (N, desc[D_NOUT], Lout), (N, desc[D_NG])


@torch.library.custom_op("cherimoya_b200::forward", mutates_args=())
def forward(x: torch.Tensor, x_ctl: Optional[torch.Tensor], packed: torch.Tensor,
            packed_offset: int, desc: List[int],
            residual_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Full Cherimoya forward on one-hot / dense input x (N, 4, L)."""
    lib = _lib.load()
    _require_cuda(x, "X")
    if x.dim() != 3 or x.shape[1] != 4:
        raise RuntimeError("cherimoya_b200: expected X of shape (N, 4, L), got {}".format(
            tuple(x.shape)))
    if x.shape[2] != desc[D_L]:
        raise RuntimeError("cherimoya_b200: sequence length mismatch")
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.contiguous()
    if desc[D_NCTL] > 0:
        if x_ctl is None:
            raise RuntimeError("cherimoya_b200: model expects control tracks")
        if x_ctl.dim() != 3 or x_ctl.shape[0] != x.shape[0] or x_ctl.shape[1] != desc[D_NCTL] \
                or x_ctl.shape[2] != x.shape[2]:
            raise RuntimeError("cherimoya_b200: expected X_ctl of shape (N, {}, L)".format(
                desc[D_NCTL]))
        x_ctl = x_ctl.to(device=x.device, dtype=torch.float32).contiguous()
    else:
        x_ctl = None
    N = x.shape[0]
    ps, cs = _out_shapes(desc, N)
    profile = torch.empty(ps, dtype=torch.float32, device=x.device)
    logcounts = torch.empty(cs, dtype=torch.float32, device=x.device)
    if N == 0:
        return profile, logcounts
    d = _desc(desc, residual_scale)
    nbytes = lib.chm_forward_workspace_bytes(ctypes.byref(d), N)
    if nbytes == 0:
        _lib.check(lib.chm_validate(ctypes.byref(d)), "forward")
    ws, off = aligned_empty(nbytes, x.device)
    st = lib.chm_forward(ctypes.byref(d), ctypes.c_void_p(packed.data_ptr() + packed_offset), N,
                         _ptr(x), _lib.INPUT_BF16 if x.dtype == torch.bfloat16 else _lib.INPUT_F32,
                         _ptr(x_ctl), _ptr(profile), _ptr(logcounts),
                         ctypes.c_void_p(ws.data_ptr() + off), nbytes, _stream(x.device))
    _lib.check(st, "forward")
    return profile, logcounts


@forward.register_fake
def _forward_fake(x, x_ctl, packed, packed_offset, desc, residual_scale):
    ps, cs = _out_shapes(desc, x.shape[0])
    return x.new_empty(ps, dtype=torch.float32), x.new_empty(cs, dtype=torch.float32)


@torch.library.custom_op("cherimoya_b200::forward_bases", mutates_args=())
def forward_bases(bases: torch.Tensor, x_ctl: Optional[torch.Tensor], packed: torch.Tensor,
                  packed_offset: int, desc: List[int],
                  residual_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Full forward on base indices (N, L) int8 in 0..3 (A, C, G, T)."""
    lib = _lib.load()
    _require_cuda(bases, "bases")
    if bases.dim() != 2 or bases.shape[1] != desc[D_L]:
        raise RuntimeError("cherimoya_b200: expected bases of shape (N, L)")
    bases = bases.to(torch.int8).contiguous()
    if desc[D_NCTL] > 0:
        if x_ctl is None:
            raise RuntimeError("cherimoya_b200: model expects control tracks")
        x_ctl = x_ctl.to(device=bases.device, dtype=torch.float32).contiguous()
    else:
        x_ctl = None
    N = bases.shape[0]
    ps, cs = _out_shapes(desc, N)
    profile = torch.empty(ps, dtype=torch.float32, device=bases.device)
    logcounts = torch.empty(cs, dtype=torch.float32, device=bases.device)
    if N == 0:
        return profile, logcounts
    d = _desc(desc, residual_scale)
    nbytes = lib.chm_forward_workspace_bytes(ctypes.byref(d), N)
    ws, off = aligned_empty(nbytes, bases.device)
    st = lib.chm_forward_bases(ctypes.byref(d), ctypes.c_void_p(packed.data_ptr() + packed_offset),
                               N, _ptr(bases), _ptr(x_ctl), _ptr(profile), _ptr(logcounts),
                               ctypes.c_void_p(ws.data_ptr() + off), nbytes,
                               _stream(bases.device))
    _lib.check(st, "forward_bases")
    return profile, logcounts


@forward_bases.register_fake
def _forward_bases_fake(bases, x_ctl, packed, packed_offset, desc, residual_scale):
    ps, cs = _out_shapes(desc, bases.shape[0])
    return (bases.new_empty(ps, dtype=torch.float32), bases.new_empty(cs, dtype=torch.float32))


# ----------------------------------------------------------------- ISM / variants
@torch.library.custom_op("cherimoya_b200::ism", mutates_args=())
def ism(bases: torch.Tensor, start: int, end: int, mutant_batch: int, packed: torch.Tensor,
        packed_offset: int, desc: List[int],
        residual_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Saturation mutagenesis of positions [start, end): returns
    d_logcount (N, n_groups, 4, W) and jsd (N, 4, W)."""
    lib = _lib.load()
    _require_cuda(bases, "bases")
    if bases.dim() != 2 or bases.shape[1] != desc[D_L]:
        raise RuntimeError("cherimoya_b200: expected bases of shape (N, L)")
    if not (0 <= start < end <= desc[D_L]):
        raise RuntimeError("cherimoya_b200: invalid ISM window [{}, {})".format(start, end))
    bases = bases.to(torch.int8).contiguous()
    N, W = bases.shape[0], end - start
    dlc = torch.empty(N, desc[D_NG], 4, W, dtype=torch.float32, device=bases.device)
    jsd = torch.empty(N, 4, W, dtype=torch.float32, device=bases.device)
    if N == 0:
        return dlc, jsd
    d = _desc(desc, residual_scale)
    mb = max(1, int(mutant_batch))
    nbytes = lib.chm_ism_workspace_bytes(ctypes.byref(d), N, mb)
    ws, off = aligned_empty(nbytes, bases.device)
    st = lib.chm_ism(ctypes.byref(d), ctypes.c_void_p(packed.data_ptr() + packed_offset), N,
                     _ptr(bases), int(start), int(end), mb, _ptr(dlc), _ptr(jsd),
                     ctypes.c_void_p(ws.data_ptr() + off), nbytes, _stream(bases.device))
    _lib.check(st, "ism")
    return dlc, jsd


@ism.register_fake
def _ism_fake(bases, start, end, mutant_batch, packed, packed_offset, desc, residual_scale):
    N, W = bases.shape[0], end - start
    return (bases.new_empty((N, desc[D_NG], 4, W), dtype=torch.float32),
            bases.new_empty((N, 4, W), dtype=torch.float32))


@torch.library.custom_op("cherimoya_b200::ism_targets", mutates_args=())
def ism_targets(bases: torch.Tensor, start: int, end: int, mutant_batch: int,
                packed: torch.Tensor, packed_offset: int, desc: List[int],
                residual_scale: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """ism() plus the change of the ProfileWrapper value in every mutant:
    d_logcount (N, n_groups, 4, W), jsd (N, 4, W), d_profile_wrapper (N, 4, W)."""
    lib = _lib.load()
    _require_cuda(bases, "bases")
    if bases.dim() != 2 or bases.shape[1] != desc[D_L]:
        raise RuntimeError("cherimoya_b200: expected bases of shape (N, L)")
    if not (0 <= start < end <= desc[D_L]):
        raise RuntimeError("cherimoya_b200: invalid ISM window [{}, {})".format(start, end))
    bases = bases.to(torch.int8).contiguous()
    N, W = bases.shape[0], end - start
    dlc = torch.empty(N, desc[D_NG], 4, W, dtype=torch.float32, device=bases.device)
    jsd = torch.empty(N, 4, W, dtype=torch.float32, device=bases.device)
    dpw = torch.empty(N, 4, W, dtype=torch.float32, device=bases.device)
    if N == 0:
        return dlc, jsd, dpw
    d = _desc(desc, residual_scale)
    mb = max(1, int(mutant_batch))
    nbytes = lib.chm_ism_workspace_bytes(ctypes.byref(d), N, mb)
    ws, off = aligned_empty(nbytes, bases.device)
    st = lib.chm_ism_ex(ctypes.byref(d), ctypes.c_void_p(packed.data_ptr() + packed_offset), N,
                        _ptr(bases), int(start), int(end), mb, _ptr(dlc), _ptr(jsd), _ptr(dpw),
                        ctypes.c_void_p(ws.data_ptr() + off), nbytes, _stream(bases.device))
    _lib.check(st, "ism_targets")
    return dlc, jsd, dpw


@ism_targets.register_fake
def _ism_targets_fake(bases, start, end, mutant_batch, packed, packed_offset, desc,
                      residual_scale):
    N, W = bases.shape[0], end - start
    return (bases.new_empty((N, desc[D_NG], 4, W), dtype=torch.float32),
            bases.new_empty((N, 4, W), dtype=torch.float32),
            bases.new_empty((N, 4, W), dtype=torch.float32))


# ----------------------------------------------------------------- wrapper epilogues
def _epilogue_desc(profile, n_groups):
    # only n_outputs, n_groups and the output length matter to the epilogues
    N, n_out, Lout = profile.shape
    return _lib.make_desc(128, 0, 1, n_out, n_groups, 0, 0, Lout, 0.0, _lib.MODE_FP32)


@torch.library.custom_op("cherimoya_b200::expected_counts", mutates_args=())
def expected_counts(profile: torch.Tensor, logcounts: torch.Tensor,
                    group_sizes: List[int]) -> torch.Tensor:
    """ExpectedCountsWrapper's output from a forward's (profile, logcounts):
    per signal group a joint softmax over its channels and positions times
    expm1(logcount), one fused kernel."""
    lib = _lib.load()
    _require_cuda(profile, "profile")
    profile = profile.float().contiguous()
    logcounts = logcounts.to(device=profile.device, dtype=torch.float32).contiguous()
    if profile.dim() != 3 or logcounts.shape != (profile.shape[0], len(group_sizes)) or \
            sum(group_sizes) != profile.shape[1]:
        raise RuntimeError("cherimoya_b200: expected_counts shape mismatch")
    out = torch.empty_like(profile)
    if profile.shape[0] == 0:
        return out
    d = _epilogue_desc(profile, len(group_sizes))
    gs = (ctypes.c_int32 * len(group_sizes))(*[int(g) for g in group_sizes])
    st = lib.chm_wrapper_epilogue(ctypes.byref(d), profile.shape[0], _ptr(profile),
                                  _ptr(logcounts), gs, _ptr(out), None, None, 0,
                                  _stream(profile.device))
    _lib.check(st, "expected_counts")
    return out


@expected_counts.register_fake
def _expected_counts_fake(profile, logcounts, group_sizes):
    return torch.empty_like(profile, dtype=torch.float32)


@torch.library.custom_op("cherimoya_b200::profile_wrapper", mutates_args=())
def profile_wrapper(profile: torch.Tensor) -> torch.Tensor:
    """ProfileWrapper's output (N, 1) from profile logits (N, n_out, Lout)."""
    lib = _lib.load()
    _require_cuda(profile, "profile")
    profile = profile.float().contiguous()
    if profile.dim() != 3:
        raise RuntimeError("cherimoya_b200: profile_wrapper expects (N, n_out, L)")
    N = profile.shape[0]
    out = torch.empty(N, 1, dtype=torch.float32, device=profile.device)
    if N == 0:
        return out
    d = _epilogue_desc(profile, 1)
    ws = torch.empty_like(profile)            # the softmax, not returned
    st = lib.chm_wrapper_epilogue(ctypes.byref(d), N, _ptr(profile), _ptr(profile), None, None,
                                  _ptr(out), _ptr(ws), ws.numel() * 4, _stream(profile.device))
    _lib.check(st, "profile_wrapper")
    return out


@profile_wrapper.register_fake
def _profile_wrapper_fake(profile):
    return profile.new_empty((profile.shape[0], 1), dtype=torch.float32)


@torch.library.custom_op("cherimoya_b200::variant", mutates_args=())
def variant(ref_bases: torch.Tensor, alt_bases: torch.Tensor, packed: torch.Tensor,
            packed_offset: int, desc: List[int],
            residual_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Ref/alt scoring: d_logcount (N, n_groups), jsd (N,)."""
    lib = _lib.load()
    _require_cuda(ref_bases, "ref_bases")
    if ref_bases.shape != alt_bases.shape or ref_bases.dim() != 2 \
            or ref_bases.shape[1] != desc[D_L]:
        raise RuntimeError("cherimoya_b200: expected ref/alt bases of equal shape (N, L)")
    ref_bases = ref_bases.to(torch.int8).contiguous()
    alt_bases = alt_bases.to(device=ref_bases.device, dtype=torch.int8).contiguous()
    N = ref_bases.shape[0]
    dlc = torch.empty(N, desc[D_NG], dtype=torch.float32, device=ref_bases.device)
    jsd = torch.empty(N, dtype=torch.float32, device=ref_bases.device)
    if N == 0:
        return dlc, jsd
    d = _desc(desc, residual_scale)
    nbytes = lib.chm_variant_workspace_bytes(ctypes.byref(d), N)
    ws, off = aligned_empty(nbytes, ref_bases.device)
    st = lib.chm_variant(ctypes.byref(d), ctypes.c_void_p(packed.data_ptr() + packed_offset), N,
                         _ptr(ref_bases), _ptr(alt_bases), _ptr(dlc), _ptr(jsd),
                         ctypes.c_void_p(ws.data_ptr() + off), nbytes, _stream(ref_bases.device))
    _lib.check(st, "variant")
    return dlc, jsd


@variant.register_fake
def _variant_fake(ref_bases, alt_bases, packed, packed_offset, desc, residual_scale):
    N = ref_bases.shape[0]
    return (ref_bases.new_empty((N, desc[D_NG]), dtype=torch.float32),
            ref_bases.new_empty((N,), dtype=torch.float32))


def last_launch_count():
    """Engine kernel launches issued by the last C-ABI call on this thread."""
    return int(_lib.load().chm_last_launch_count())


# ----------------------------------------------------------------- one block
def pack_block(conv_weight, linear1_weight, linear2_weight, residual_scale, device):
    """Pack one Cheri Block's weights; returns (buffer, offset)."""
    lib = _lib.load()
    C, H = int(linear1_weight.shape[1]), int(linear1_weight.shape[0])
    nbytes = lib.chm_block_packed_bytes(C, H)
    if nbytes == 0:
        raise RuntimeError("cherimoya_b200: unsupported block shape C={} H={}".format(C, H))
    buf, off = aligned_empty(nbytes, device)
    ts = [t.detach().to(device=device, dtype=torch.float32).contiguous()
          for t in (conv_weight, linear1_weight, linear2_weight)]
    st = lib.chm_pack_block(C, H, float(residual_scale), _ptr(ts[0]), _ptr(ts[1]), _ptr(ts[2]),
                            ctypes.c_void_p(buf.data_ptr() + off), nbytes, _stream(device))
    _lib.check(st, "pack_block")
    torch.cuda.current_stream(device).synchronize()
    return buf, off


@torch.library.custom_op("cherimoya_b200::block_forward", mutates_args=())
def block_forward(x: torch.Tensor, packed: torch.Tensor, packed_offset: int, hidden: int,
                  dilation: int) -> torch.Tensor:
    """One Cheri Block on x (N, L, C) fp32 or bf16."""
    lib = _lib.load()
    _require_cuda(x, "X")
    if x.dim() != 3:
        raise RuntimeError("cherimoya_b200: expected (N, L, C), got {}".format(tuple(x.shape)))
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.contiguous()
    N, L, C = x.shape
    out = torch.empty_like(x)
    if N == 0:
        return out
    dt = _lib.INPUT_BF16 if x.dtype == torch.bfloat16 else _lib.INPUT_F32
    nbytes = lib.chm_block_workspace_bytes(N, L, C, dt)
    ws, off = aligned_empty(nbytes, x.device)
    st = lib.chm_block_forward(N, L, C, int(hidden), int(dilation), dt,
                               ctypes.c_void_p(packed.data_ptr() + packed_offset), _ptr(x),
                               _ptr(out), ctypes.c_void_p(ws.data_ptr() + off), nbytes,
                               _stream(x.device))
    _lib.check(st, "block_forward")
    return out


@block_forward.register_fake
def _block_forward_fake(x, packed, packed_offset, hidden, dilation):
    return torch.empty_like(x)
