"""bf16 operand copies of fp32 master weights, made once per optimizer step.

The tcgen05 GEMMs read bf16 operands; the parameters stay fp32.  Instead of casting (and, in
backward, transposing) every weight at every call, :func:`bf16` / :func:`bf16_t` /
:func:`pair_bf16` return a cached copy that is rebuilt only when the parameter may have
changed.  A cached copy is keyed by

* a global epoch, advanced after every ``torch.optim`` optimizer step (a process-wide
  step post-hook; fused optimizers update parameters without bumping their version
  counters, so the epoch is what catches their updates),
* the parameter's version counter (in-place edits such as ``load_state_dict``),
* its storage address,

and holds a weak reference to the parameter itself (an entry is dropped when its parameter dies).

On the kernel path the copies are written by the ``weight_pack`` kernel, and the optimizer-step
hook rewrites every live entry in place with one launch per 48 entries (the new epoch, version
and unchanged storage address become the entry's key), instead of dropping the cache and
rebuilding each copy on its next use with several small launches.

Code that changes weights some other way (through ``.data``) calls :func:`invalidate`.
"""

from __future__ import annotations

import weakref

import torch

_EPOCH = [0]
_CACHE: dict[int, tuple] = {}


# weight_pack job kinds (``maloq::kPack*``)
_KIND = {"bf16": 0, "bf16_t": 1, "pair": 2, "pair_t": 3}
_PAIR_GRAD = 4


def _kernel_path(t):
    from maloq_b200 import ops

    return ops._cuda(t)


def _lib():
    from .kernels import lib

    return lib()


def _packable(w, kind):
    """True when ``weight_pack`` can write the ``kind`` copy of ``w`` (the kernel path's case)."""
    if kind not in _KIND or w.dtype != torch.float32 or not w.is_contiguous():
        return False
    if not (1 if kind == "bf16" else 2) <= w.dim() <= (2 if kind in ("pair", "pair_t") else 3):
        return False
    if kind in ("pair", "pair_t") and w.shape[0] % 2:
        return False
    return _kernel_path(w)


def _out_shape(p, kind):
    if kind == "bf16":
        return tuple(p.shape)
    if kind == "bf16_t":
        return tuple(p.shape[:-2]) + (p.shape[-1], p.shape[-2])
    if kind == "pair":
        return (p.shape[0], 2 * p.shape[1])
    return (2 * p.shape[1], p.shape[0])  # pair_t


def _refresh():
    """Rewrite every live kernel-path entry from its (updated) parameter in place; entries whose
    parameter died, moved or is off the kernel path are dropped."""
    from .native import count_launches

    srcs, dsts, kinds, keep = [], [], [], {}
    for k, (key, t, ref) in list(_CACHE.items()):
        p = ref()
        if p is None or p.data_ptr() != key[2] or p.device != t.device or not _packable(p.detach(), k[1]):
            continue
        srcs.append(p.detach())
        dsts.append(t)
        kinds.append(_KIND[k[1]])
        keep[k] = (p, t, ref)
    _CACHE.clear()
    if srcs:
        _lib().weight_pack(srcs, dsts, kinds)
        count_launches(-(-len(srcs) // 48))
    for k, (p, t, ref) in keep.items():
        _CACHE[k] = ((_EPOCH[0], p._version, p.data_ptr(), k[1]), t, ref)


def _bump(*_args, **_kwargs):
    _EPOCH[0] += 1
    _refresh()


from torch.optim.optimizer import register_optimizer_step_post_hook  # noqa: E402

register_optimizer_step_post_hook(_bump)


def invalidate() -> None:
    """Drop every cached copy (call after changing weights through ``.data``)."""
    _EPOCH[0] += 1
    _CACHE.clear()


def _get(p, kind, make):
    if not isinstance(p, torch.nn.Parameter):  # only parameters live long enough to cache
        return make(p.detach())
    key = (_EPOCH[0], p._version, p.data_ptr(), kind)
    ent = _CACHE.get((id(p), kind))
    # the entry must belong to this very parameter: a freed parameter's id and storage address
    # can be reused by a new one with the same version count (e.g. a model built after another
    # was deleted), which the key alone would not tell apart
    if ent is not None and ent[0] == key and ent[2]() is p:
        return ent[1]
    w = p.detach()
    if _packable(w, kind):
        from .native import count_launches

        t = torch.empty(_out_shape(w, kind), device=w.device, dtype=torch.bfloat16)
        _lib().weight_pack([w], [t], [_KIND[kind]])
        count_launches(1)
    else:
        t = make(w)
    _CACHE[(id(p), kind)] = (key, t, weakref.ref(p, lambda _r, k=(id(p), kind): _CACHE.pop(k, None)))
    return t


def bf16(p):
    """Contiguous bf16 copy of ``p``."""
    return _get(p, "bf16", lambda w: w.to(torch.bfloat16).contiguous())


def bf16_t(p):
    """Contiguous bf16 copy of the transpose of a 2-D ``p`` (or of each matrix of a 3-D one)."""
    return _get(p, "bf16_t", lambda w: bf16(p).transpose(-1, -2).contiguous() if isinstance(p, torch.nn.Parameter)
                else w.transpose(-1, -2).to(torch.bfloat16).contiguous())


def _pair(w):
    """[[W_r, -W_i], [W_i, W_r]] of w = [W_r; W_i]: rows r of the result interleave the blocks
    as [W_r[r] | -W_i[r]] and [W_i[r] | W_r[r]]."""
    h, k = w.shape[0] // 2, w.shape[1]
    wr, wi = w[:h], w[h:]
    return torch.stack([torch.stack([wr, -wi], 1), torch.stack([wi, wr], 1)], 0).view(2 * h, 2 * k)


def pair_bf16(p):
    """bf16 [[W_r, -W_i], [W_i, W_r]] of an SO(2) m > 0 weight ``p`` = [W_r; W_i]."""
    return _get(p, "pair", lambda w: _pair(w).to(torch.bfloat16).contiguous())


def pair_bf16_t(p):
    # the transpose of the cached pair matrix: one copy instead of rebuilding the blocks
    return _get(p, "pair_t", lambda w: pair_bf16(p).t().contiguous() if isinstance(p, torch.nn.Parameter)
                else _pair(w).t().to(torch.bfloat16).contiguous())


def pair_grad(dP):
    """Gradient of ``p`` = [W_r; W_i] from the gradient of its pair matrix."""
    h2, k2 = dP.shape
    d = dP.view(2, h2 // 2, 2, k2 // 2)
    return torch.cat([d[0, :, 0] + d[1, :, 1], d[1, :, 0] - d[0, :, 1]], 0)


def pair_grads(dPs):
    """:func:`pair_grad` of each fp32 pair-matrix gradient, in one launch on the kernel path."""
    if not dPs:
        return []
    if not all(d.dtype == torch.float32 and d.is_contiguous() and d.dim() == 2 and d.shape[0] % 2 == 0
               and d.shape[1] % 2 == 0 and _kernel_path(d) for d in dPs):
        return [pair_grad(d) for d in dPs]
    from .native import count_launches

    outs = [torch.empty(d.shape[0], d.shape[1] // 2, device=d.device, dtype=torch.float32) for d in dPs]
    _lib().weight_pack(list(dPs), outs, [_PAIR_GRAD] * len(dPs))
    count_launches(-(-len(dPs) // 48))
    return outs
