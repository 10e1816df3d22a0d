"""Loss functions, optimizers and schedulers (reference ``train_utils/loss.py``).

Names and semantics of the reference's loss functions are kept so that configs naming
them keep working.  ``*_padded`` losses average over all given entries (callers pass
already-masked tensors); ``*_unpadded`` losses mask ``target != 0`` themselves.
On CUDA the fused masked-loss kernel computes the Fock loss and its gradient in one pass
(:func:`maloq_b200.ops.loss.fock_loss`).
"""

from __future__ import annotations

import torch
import torch.nn as nn


def mse_padded_loss(output, target, req_irreps=None):
    return nn.functional.mse_loss(output, target)


def l1_padded_loss(output, target, req_irreps=None):
    return nn.functional.l1_loss(output, target)


def rmse_padded_loss(output, target, req_irreps=None):
    return torch.sqrt(nn.functional.mse_loss(output, target))


def rmse_mse_padded_loss(output, target, req_irreps=None):
    mse = nn.functional.mse_loss(output, target)
    return torch.sqrt(mse) + mse


def combined_padded_loss(output, target, req_irreps=None):
    return torch.sqrt(nn.functional.mse_loss(output, target)) + nn.functional.l1_loss(output, target)


def _masked_mean(err, mask):
    return (err * mask).sum() / mask.sum()


def mse_unpadded_loss(output, target, req_irreps=None):
    return _masked_mean((output - target) ** 2, (target != 0).to(output.dtype))


def l1_unpadded_loss(output, target, req_irreps=None):
    return _masked_mean((output - target).abs(), (target != 0).to(output.dtype))


def combined_unpadded_loss(output, target, req_irreps=None):
    m = (target != 0).to(output.dtype)
    return _masked_mean((output - target) ** 2, m) + _masked_mean((output - target).abs(), m)


def weighted_irrep_mse_loss(output, target, req_irreps, weights=None):
    """Mean over irreps of the per-irrep MSE (each irrep weighted 1)."""
    ls = [it.l for it in req_irreps for _ in range(it.mul)] if hasattr(req_irreps, "__iter__") else req_irreps.ls
    weights = weights or [1.0] * len(ls)
    tot, wsum, p = 0.0, 0.0, 0
    for l, w in zip(ls, weights):
        d = 2 * l + 1
        tot = tot + w * nn.functional.mse_loss(output[:, p:p + d], target[:, p:p + d])
        wsum += w
        p += d
    return tot / wsum


def geometric_mean_loss(output, target, req_irreps=None):
    return torch.exp(torch.mean(torch.log(torch.abs(output - target))))


LOSSES = {f.__name__: f for f in (mse_padded_loss, l1_padded_loss, rmse_padded_loss, rmse_mse_padded_loss,
                                   combined_padded_loss, mse_unpadded_loss, weighted_irrep_mse_loss,
                                   l1_unpadded_loss, geometric_mean_loss, combined_unpadded_loss)}


def get_loss(name_or_fn):
    if callable(name_or_fn):
        return name_or_fn
    return LOSSES[name_or_fn]


# ------------------------------------------------------------------ Muon
def zeropower_via_newtonschulz5(G, steps: int = 5):
    """Orthogonalise G with the quintic Newton-Schulz iteration (a, b, c) =
    (3.4445, -4.7750, 2.0315) from the Muon optimizer (K. Jordan et al., 2024), in bf16."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.bfloat16()
    transposed = G.size(-2) > G.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    if transposed:
        X = X.mT
    return X


def _muon_update(p, st, lr, momentum, nesterov, ns_steps, weight_decay):
    """One Muon step of parameter ``p`` (state ``st``): momentum, the Newton-Schulz orthogonalised
    update of the [rows, rest] matrix scaled by sqrt(max(1, rows / cols)), decoupled decay."""
    buf = st.setdefault("momentum_buffer", torch.zeros_like(p))
    buf.mul_(momentum).add_(p.grad)
    upd = p.grad.add(buf, alpha=momentum) if nesterov else buf
    shape = upd.shape
    u = zeropower_via_newtonschulz5(upd.reshape(shape[0], -1), ns_steps).to(p.dtype)
    u = u.reshape(shape) * max(1.0, shape[0] / max(1, u[0].numel())) ** 0.5
    if weight_decay:
        p.mul_(1 - lr * weight_decay)
    p.add_(u, alpha=-lr)


class Muon(torch.optim.Optimizer):
    """Muon alone, for parameters of two or more dimensions (reference ``train_utils/loss.py:164-208``;
    reference default: no Nesterov momentum)."""

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=False, ns_steps=5, weight_decay=0.0):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                                      weight_decay=weight_decay))
        for g in self.param_groups:
            for p in g["params"]:
                if p.ndim < 2:
                    raise ValueError(f"Muon updates matrices only; got a parameter of shape {tuple(p.shape)} "
                                     "(use HybridMuon for mixed parameter sets)")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is not None:
                    _muon_update(p, self.state[p], g["lr"], g["momentum"], g["nesterov"], g["ns_steps"],
                                 g["weight_decay"])
        return loss


class HybridMuon(torch.optim.Optimizer):
    """Muon (momentum + Newton-Schulz orthogonalised update) for >= 2-D parameters and
    AdamW for the rest (reference ``train_utils/loss.py:164-248``)."""

    def __init__(self, params, muon_lr=0.02, adamw_lr=1e-4, momentum=0.95, nesterov=True, ns_steps=5,
                 betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        params = list(params)
        muon = [p for p in params if p.ndim >= 2]
        adam = [p for p in params if p.ndim < 2]
        groups = []
        if muon:
            groups.append(dict(params=muon, use_muon=True, lr=muon_lr, momentum=momentum, nesterov=nesterov,
                               ns_steps=ns_steps, weight_decay=weight_decay, betas=betas, eps=eps))
        if adam:
            groups.append(dict(params=adam, use_muon=False, lr=adamw_lr, betas=betas, eps=eps,
                               weight_decay=weight_decay, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps))
        super().__init__(groups, {})

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if g["use_muon"]:
                    _muon_update(p, st, g["lr"], g["momentum"], g["nesterov"], g["ns_steps"], g["weight_decay"])
                else:
                    st.setdefault("step", 0)
                    st["step"] += 1
                    m = st.setdefault("exp_avg", torch.zeros_like(p))
                    v = st.setdefault("exp_avg_sq", torch.zeros_like(p))
                    b1, b2 = g["betas"]
                    m.mul_(b1).add_(p.grad, alpha=1 - b1)
                    v.mul_(b2).addcmul_(p.grad, p.grad, value=1 - b2)
                    mh = m / (1 - b1 ** st["step"])
                    vh = v / (1 - b2 ** st["step"])
                    if g["weight_decay"]:
                        p.mul_(1 - g["lr"] * g["weight_decay"])
                    p.addcdiv_(mh, vh.sqrt().add_(g["eps"]), value=-g["lr"])


class MonotonicDecreaseScheduler:
    """Halve the LR whenever the validation loss does not improve (``loss.py:253-284``)."""

    def __init__(self, optimizer, factor=0.5, min_lr=1e-10):
        self.optimizer, self.factor, self.min_lr, self.best = optimizer, factor, min_lr, float("inf")

    def step(self, val_loss):
        if val_loss < self.best:
            self.best = val_loss
            return
        for g in self.optimizer.param_groups:
            g["lr"] = max(self.min_lr, g["lr"] * self.factor)


def adjust_learning_rate(optimizer, epoch, warmup_epochs, initial_lr, final_lr):
    if epoch < warmup_epochs:
        lr = initial_lr + (final_lr - initial_lr) * (epoch / warmup_epochs)
        for g in optimizer.param_groups:
            g["lr"] = lr
