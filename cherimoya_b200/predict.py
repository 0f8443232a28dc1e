"""Batched inference over a large set of examples, and reverse-complement
averaging.

Upstream calls ``tangermeme.predict.predict(model, X, args=..., batch_size=...,
device=..., dtype=...)`` for every bulk prediction (``cherimoya/cherimoya.py:567-568``,
``cherimoya_cli/commands/evaluate.py:70-78``) and averages the forward and
reverse-complement strands in ``cherimoya_cli/commands/evaluate.py:80-96``.
``predict`` keeps that call shape: X and every tensor in ``args`` are cut
into batches along the first dimension, each batch goes through
``model(X_batch, *args_batch)`` under ``no_grad``, and the outputs are
concatenated on the host in input order.

On a CUDA device the host side is pipelined: batch k+1 is copied to the
device on a second stream while batch k computes, and batch k's outputs
are copied back on the same stream while batch k+1 computes. Host inputs
that are not in pinned memory pass through two pinned staging buffers of
one batch each, so host memory grows by two batches, not by a copy of X.

``dtype`` names the arithmetic: "float32" runs the engine's fp32 mode,
"bfloat16" runs the model under bf16 autocast, which selects the engine's
bf16 mode on CUDA and upstream's CPU autocast path on the CPU. A model
built with ``precision="fp32"`` or ``"bf16"`` keeps its own mode.
"""

import torch

_DTYPES = {
    "float32": torch.float32, "float": torch.float32, "fp32": torch.float32,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
    torch.float32: torch.float32, torch.bfloat16: torch.bfloat16,
}


def _arith_dtype(dtype):
    if dtype is None:
        return torch.float32
    if dtype not in _DTYPES:
        raise ValueError("dtype must be 'float32' or 'bfloat16', got {!r}".format(dtype))
    return _DTYPES[dtype]


def _as_tuple(out):
    return (out,) if isinstance(out, torch.Tensor) else tuple(out)


def rc_forward(model, X, *args):
    """(profile, logcounts) averaged over X and its reverse complement, as
    upstream ``cherimoya_cli/commands/evaluate.py:80-96`` does: the reverse
    complement flips the base axis and the position axis of X (and of each
    control track), its profile is flipped back over channels and positions,
    and both outputs are averaged with the forward strand's. Both strands run
    as one forward of a doubled batch."""
    n = X.shape[0]
    out = _as_tuple(model(torch.cat([X, X.flip(-1, -2)]),
                          *[torch.cat([a, a.flip(-1, -2)]) for a in args]))
    if len(out) != 2:
        raise RuntimeError("reverse-complement averaging needs a (profile, logcounts) model")
    y, c = out
    return (y[:n] + y[n:].flip(-1, -2)) / 2, (c[:n] + c[n:]) / 2


def _run_batch(model, xb, eb, rc):
    return _as_tuple(rc_forward(model, xb, *eb) if rc else model(xb, *eb))


def predict(model, X, args=None, batch_size=64, device="cuda", dtype="float32", verbose=False,
            reverse_complement_average=False):
    """Outputs of ``model`` over all examples of X, batch by batch.

    X: (N, 4, L) tensor on the host or on ``device``; args: None or a tuple
    of per-example tensors passed after X (control tracks). Returns the
    model's outputs concatenated over batches as host tensors (in pinned
    memory when ``device`` is a GPU): a tuple when the model returns a
    tuple, else one tensor. With ``reverse_complement_average`` the model
    must return (profile, logcounts) and both strands are averaged
    (``rc_forward``).
    """
    extra = tuple(args) if args is not None else ()
    for a in extra:
        if a.shape[0] != X.shape[0]:
            raise ValueError("every tensor in args needs X's first dimension")
    if batch_size < 1:
        raise ValueError("batch_size must be positive")
    arith = _arith_dtype(dtype)
    dev = torch.device(device)
    N = X.shape[0]
    batches = [(s, min(s + batch_size, N)) for s in range(0, N, batch_size)]
    if not batches:
        raise ValueError("predict needs at least one example")
    progress = None
    if verbose:
        from tqdm import tqdm
        progress = tqdm(total=len(batches))
    autocast = torch.autocast(dev.type, dtype=torch.bfloat16, enabled=arith == torch.bfloat16)
    with torch.no_grad(), autocast:
        if dev.type != "cuda":
            cols = []
            for s, e in batches:
                cols.append(_run_batch(model, X[s:e].to(dev), [a[s:e].to(dev) for a in extra],
                                       reverse_complement_average))
                if progress is not None:
                    progress.update(1)
            res = tuple(torch.cat([c[i].cpu() for c in cols]) for i in range(len(cols[0])))
        else:
            res = _predict_cuda(model, X, extra, batches, dev, reverse_complement_average,
                                progress)
    if progress is not None:
        progress.close()
    return res[0] if len(res) == 1 else res


def _predict_cuda(model, X, extra, batches, dev, rc, progress):
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    srcs = (X,) + extra
    resident = all(t.device == dev for t in srcs)
    compute = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(device=dev)
    copy.wait_stream(compute)      # buffers the allocator hands out below are free on both
    bmax = max(e - s for s, e in batches)

    if resident:
        def stage(b, s, e):
            return [t[s:e] for t in srcs]
    else:
        srcs = tuple(t.contiguous() for t in srcs)
        on_dev = [t.device == dev for t in srcs]
        # inputs on another GPU copy device to device, without host staging
        pinned = [d or t.is_cuda or t.is_pinned() for t, d in zip(srcs, on_dev)]
        # two device buffers (and, for pageable host inputs, two pinned host
        # buffers) per input not already on the device, used by alternate batches
        dbuf = [[None if d else torch.empty((bmax,) + tuple(t.shape[1:]), dtype=t.dtype,
                                            device=dev)
                 for t, d in zip(srcs, on_dev)] for _ in range(2)]
        hbuf = [[None if p else torch.empty((bmax,) + tuple(t.shape[1:]), dtype=t.dtype,
                                            pin_memory=True)
                 for t, p in zip(srcs, pinned)] for _ in range(2)]
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]

        def stage(b, s, e):
            if used[b]:
                h2d_done[b].synchronize()       # the pinned buffer's last copy has left
            with torch.cuda.stream(copy):
                if used[b]:
                    copy.wait_event(consumed[b])   # the device buffer's last batch is done
                out = []
                for t, d, h in zip(srcs, dbuf[b], hbuf[b]):
                    src = t[s:e]
                    if d is None:
                        out.append(src)
                        continue
                    if h is not None:
                        h[:e - s].copy_(src)
                        src = h[:e - s]
                    d[:e - s].copy_(src, non_blocking=True)
                    out.append(d[:e - s])
                h2d_done[b].record(copy)
            used[b] = True
            return out

    host_out = None
    staged = stage(0, *batches[0])
    for k, (s, e) in enumerate(batches):
        cur = staged
        if not resident:
            compute.wait_event(h2d_done[k % 2])
        outs = _run_batch(model, cur[0], cur[1:], rc)
        if not resident:
            consumed[k % 2].record(compute)
        if host_out is None:
            host_out = [torch.empty((batches[-1][1],) + tuple(o.shape[1:]), dtype=o.dtype,
                                    pin_memory=True) for o in outs]
        if k + 1 < len(batches):
            ns, ne = batches[k + 1]
            staged = stage((k + 1) % 2, ns, ne)   # overlaps batch k's compute
        done = torch.cuda.Event()
        done.record(compute)
        with torch.cuda.stream(copy):
            copy.wait_event(done)
            for h, o in zip(host_out, outs):
                o.record_stream(copy)
                h[s:e].copy_(o, non_blocking=True)
        if progress is not None:
            progress.update(1)
    copy.synchronize()
    compute.synchronize()
    return tuple(host_out)
