"""Synthetic datasets of the benchmark configurations (no datasets are available offline).

``build_dataset(name, n, ...)`` returns graph samples with coupled-basis Fock targets from
a frozen random-init teacher (:class:`maloq_b200.data.targets.Teacher`).  Names:

==================  ===============================================  ==============  ======
name                structures                                       basis           cutoff
==================  ===============================================  ==============  ======
``small``           3-9 atoms {H,C,N,O}, 4 A cube, dmin 0.9 A         split_valence   5 A
``druglike``        30-50 atoms, bonded chains/rings                 def2_svp_like   6 A
``large``           10-150 atoms                                     def2_tzvp_like  6 A
``sio2``            amorphous Si/O, periodic                         dzvp_like       8 A
``slab``            Si slab + Hf/O oxide layer (inference only)      dzvp_like       8 A
==================  ===============================================  ==============  ======
"""

from __future__ import annotations

import numpy as np
import torch

from . import basis_sets, structures
from .batch import make_sample
from .targets import FockLabeler, Teacher, attach_targets

SPECS = {
    "small": dict(basis="split_valence_small", cutoff=5.0, gen=lambda r: structures.random_small_molecule(r)),
    "druglike": dict(basis="def2_svp_like", cutoff=6.0, gen=lambda r: structures.random_druglike_molecule(r)),
    "large": dict(basis="def2_tzvp_like", cutoff=6.0, gen=lambda r: structures.random_large_molecule(r)),
    "sio2": dict(basis="dzvp_like", cutoff=8.0, gen=None),
    "slab": dict(basis="dzvp_like", cutoff=8.0, gen=None),
}


def labeler_for(name, device="cpu"):
    return FockLabeler(basis_sets.get_basis(SPECS[name]["basis"]), device=device)


def build_samples(name, n, seed=0, cutoff=None, **kw):
    spec = SPECS[name]
    rng = np.random.default_rng(seed)
    cutoff = spec["cutoff"] if cutoff is None else cutoff
    if name == "sio2":
        return [make_sample(structures.amorphous_sio2(rng, kw.get("n_atoms", 20000)), cutoff) for _ in range(n)]
    if name == "slab":
        return [make_sample(structures.si_slab_with_oxide(rng, kw.get("n_atoms", 1_000_000)), cutoff) for _ in range(n)]
    return [make_sample(spec["gen"](rng), cutoff) for _ in range(n)]


def build_dataset(name, n, model_kwargs, seed=0, device="cpu", teacher_seed=1234, cutoff=None, labeler=None,
                  target="fock_matrix", **kw):
    """Samples with targets.  ``model_kwargs`` size the teacher (same architecture as the
    trained model: lmax/mmax/channels/layers/basis count).  ``target``: Fock labels
    (``fock_matrix`` / ``density_matrix``), or teacher ``energies`` / ``forces``."""
    labeler = labeler or labeler_for(name, device)
    samples = build_samples(name, n, seed, cutoff, **kw)
    teacher = Teacher(model_kwargs, labeler, seed=teacher_seed, device=device)
    if target in ("energies", "forces"):
        from .targets import attach_scalar_targets

        attach_scalar_targets(samples, teacher, target)
    else:
        hs = teacher.hamiltonians(samples)
        attach_targets(samples, hs, labeler)
    del teacher
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return samples, labeler
