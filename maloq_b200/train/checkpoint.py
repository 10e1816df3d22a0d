"""Checkpoints in the reference layout plus resume state.

Files written to ``output_folder`` (reference ``splittrainer.py:1828-1872``):

* ``backbone.pt`` / ``head.pt``: ``{'model_state_dict', 'optimizer_state_dict'}``;
* ``backbone_state_dic.pt`` / ``head_state_dic.pt``: the raw state dicts;
* ``{backbone|head}_training_loss.txt`` / ``_validation_loss.txt``: ``edge\\tnode`` per epoch;
* ``loss.png``: the four loss curves on a log scale (``maloq_b200.utils.lossplot``);
* ``resume.pt`` (new): epoch, scheduler state, loss history and RNG states, so a restart
  continues at the next epoch instead of epoch 0.

Writes go to a temporary file first and are renamed, so a crash never leaves a truncated
checkpoint behind.
"""

from __future__ import annotations

import os
import random

import numpy as np
import torch


def _atomic_save(obj, path):
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _unwrap(m):
    return getattr(m, "module", m)


def save_training_state(folder, backbone, head, optimizer, scheduler, epoch, history):
    os.makedirs(folder, exist_ok=True)
    for name, model in (("backbone", backbone), ("head", head)):
        model = _unwrap(model)
        if any(p.requires_grad for p in model.parameters()):
            _atomic_save({"model_state_dict": model.state_dict(), "optimizer_state_dict": optimizer.state_dict()},
                         os.path.join(folder, f"{name}.pt"))
            _atomic_save(model.state_dict(), os.path.join(folder, f"{name}_state_dic.pt"))
        with open(os.path.join(folder, f"{name}_training_loss.txt"), "w") as f:
            for e, n in zip(history["train_edge"], history["train_node"]):
                f.write(f"{e:.10f}\t{n:.10f}\n")
        with open(os.path.join(folder, f"{name}_validation_loss.txt"), "w") as f:
            for e, n in zip(history["val_edge"], history["val_node"]):
                f.write(f"{e:.10f}\t{n:.10f}\n")
    from ..utils.lossplot import save_loss_png

    save_loss_png(os.path.join(folder, "loss.png"), history)
    state = {"epoch": epoch, "history": history,
             "scheduler": scheduler.state_dict() if scheduler is not None else None,
             "rng": {"torch": torch.get_rng_state(), "numpy": np.random.get_state(), "python": random.getstate(),
                     "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}}
    _atomic_save(state, os.path.join(folder, "resume.pt"))


IGNORED_KEYS = ("output_mask",)


def load_model(model, path, device="cpu", optimizer=None):
    """Load a ``{model_state_dict, optimizer_state_dict}`` file (``module.`` prefixes stripped).

    Keys must match exactly except buffers that only one side defines among
    ``IGNORED_KEYS`` (shape bookkeeping buffers of e3nn-style linears).
    """
    ck = torch.load(path, map_location=device, weights_only=False)
    sd = ck["model_state_dict"] if "model_state_dict" in ck else ck
    sd = {k.replace("module.", ""): v for k, v in sd.items()}
    own = _unwrap(model).state_dict()
    sd = {k: v for k, v in sd.items() if k in own or not k.endswith(IGNORED_KEYS)}
    missing = [k for k in own if k not in sd and not k.endswith(IGNORED_KEYS)]
    unexpected = [k for k in sd if k not in own]
    if missing or unexpected:
        raise KeyError(f"checkpoint mismatch: missing={missing[:8]} unexpected={unexpected[:8]}")
    for k in own:
        if k not in sd:
            sd[k] = own[k]
    _unwrap(model).load_state_dict(sd, strict=True)
    if optimizer is not None and "optimizer_state_dict" in ck:
        optimizer.load_state_dict(ck["optimizer_state_dict"])
    return ck


def load_resume(folder, scheduler=None):
    path = os.path.join(folder, "resume.pt")
    if not os.path.exists(path):
        return None
    st = torch.load(path, weights_only=False)
    if scheduler is not None and st.get("scheduler") is not None:
        scheduler.load_state_dict(st["scheduler"])
    r = st["rng"]
    torch.set_rng_state(r["torch"])
    np.random.set_state(r["numpy"])
    random.setstate(r["python"])
    if r.get("cuda") is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(r["cuda"])
    return st
