"""OMol-CSH-58k Hamiltonian dataset (HDF5 + JSON key manifest) and its ORCA order fix.

File layout (reference ``dataset_utils/omol_csh_58k_dataset_utils.py:68-158``): one HDF5
group per molecule with datasets ``fock`` (the upper triangle, row-major, flattened),
``elements`` (Z) and ``coords`` (Angstrom) and attributes ``charge`` / ``spin``; a manifest
``<file>.keys.json`` lists the group names in dataset order, so a rank can open only its
slice without walking the file.

The stored Fock matrices were converted from ORCA's order with an l-sorted shell list
instead of the real def2-TZVPD shell order (diffuse shells come after the polarisation
shells).  :func:`restore_orca_diffuse_order` undoes that conversion with the l-sorted list
and redoes it with the true shell order (reference ``:11-66``).

Reading HDF5 needs ``h5py``.  It is not installed offline here, so :class:`OMolCSH58kDatabase`
takes an ``opener`` (any callable returning a mapping ``key -> group`` with array-like
members and an ``attrs`` dict); the default opener imports ``h5py`` and raises a clear error
when it is missing.  The manifest builder and the order fix are plain numpy.
"""

from __future__ import annotations

import json
import os

import numpy as np

from .readers import SYMBOL_TO_Z, reorder_orbitals, reorder_orbitals_inverse

# def2-TZVPD shell angular momenta per element (basis-set fact; diffuse shells follow the
# decrease of l), elements without two diffuse levels or g functions
DEF2_TZVPD = {
    "H": [0, 0, 0, 1, 1], "He": [0, 0, 0, 1, 1], "Li": [0, 0, 0, 0, 0, 1, 1, 1, 1],
    "Be": [0, 0, 0, 0, 0, 1, 1, 1, 2, 1], "B": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 2],
    "C": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 2], "N": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 2],
    "O": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 1, 2], "F": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 1, 2],
    "Ne": [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3, 0, 1, 2], "Na": [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 1],
    "Mg": [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 1], "Al": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 2],
    "Si": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 2], "P": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 2],
    "S": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 1, 2], "Cl": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 1, 2],
    "Ar": [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 3, 0, 1, 2], "K": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2],
    "Ca": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2],
    "Ga": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 2],
    "Ge": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 2],
    "As": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 2],
    "Se": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 1, 2],
    "Br": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 1, 2],
    "Kr": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 2, 3, 0, 1, 2],
    "Rb": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2], "Sr": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2],
    **{el: [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 3]
       for el in ("Y", "Zr", "Nb", "Mo", "Tc", "Ru", "Rh", "Pd", "Ag", "Cd", "Ba")},
    **{el: [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 3, 3, 0, 2] for el in ("In", "Sn", "Sb", "Tl", "Pb", "Bi")},
    **{el: [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 3, 3, 0, 1, 2] for el in ("Te", "I", "Xe", "Po", "At")},
    "Cs": [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2],
    **{el: [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 3, 1] for el in ("Hf", "Ta", "W", "Re", "Os", "Ir", "Pt", "Au")},
    "Hg": [0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 2, 2, 2, 3, 1],
}


def def2_tzvpd_by_z():
    """The def2-TZVPD table keyed by atomic number."""
    return {SYMBOL_TO_Z[el]: list(v) for el, v in DEF2_TZVPD.items()}


def reinflate_symmetric(flat):
    """Full symmetric matrix from its row-major upper triangle (diagonal included)."""
    flat = np.asarray(flat)
    n = int((np.sqrt(8 * len(flat) + 1) - 1) // 2)
    if n * (n + 1) // 2 != len(flat):
        raise ValueError(f"{len(flat)} values are not the upper triangle of a square matrix")
    m = np.zeros((n, n), dtype=flat.dtype)
    m[np.triu_indices(n)] = flat
    return m + m.T - np.diag(m.diagonal())


def restore_orca_diffuse_order(H, z, basis=None):
    """Fix a Fock matrix that was converted from ORCA order with l-sorted shells: convert
    back to ORCA order with the l-sorted shell list, then forward with the true shell order.
    ``H`` is square (or a flat upper triangle); ``basis`` maps Z -> shell list (default
    def2-TZVPD)."""
    basis = def2_tzvpd_by_z() if basis is None else {int(k): list(v) for k, v in basis.items()}
    H = np.asarray(H)
    if H.ndim == 1:
        H = reinflate_symmetric(H)
    z = [int(a) for a in z]
    sorted_basis = {a: sorted(basis[a]) for a in set(z)}
    raw = reorder_orbitals_inverse(H, z, sorted_basis, "orca")
    return reorder_orbitals(raw, z, basis, "orca")


def save_keys_manifest(h5path, keys=None, opener=None):
    """Write ``<h5path>.keys.json`` listing the file's top-level groups (sorted) or ``keys``."""
    if keys is None:
        f = (opener or _h5_open)(h5path)
        keys = sorted(f.keys())
    with open(f"{h5path}.keys.json", "w") as fh:
        json.dump(list(keys), fh)
    return list(keys)


def _h5_open(path):
    try:
        import h5py
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError("reading OMol-CSH HDF5 files needs h5py, which is not installed") from e
    return h5py.File(path, "r", rdcc_nbytes=64 * 1024 * 1024)


class OMolCSH58kDatabase:
    """Molecules of an OMol-CSH HDF5 file, in manifest order (``indices`` keeps a subset, e.g.
    one rank's slice).  Items: ``z``, ``pos``, ``fock`` (corrected order, float32),
    ``charge``, ``spin``, ``name``."""

    def __init__(self, dbpath, indices=None, opener=None):
        self.dbpath, self._opener, self._file = dbpath, opener or _h5_open, None
        manifest = f"{dbpath}.keys.json"
        if not os.path.exists(manifest):
            raise FileNotFoundError(f"key manifest {manifest} not found (write it with save_keys_manifest)")
        with open(manifest) as fh:
            keys = json.load(fh)
        self.keys = [keys[i] for i in indices] if indices is not None else keys

    def _f(self):
        if self._file is None:
            self._file = self._opener(self.dbpath)
        return self._file

    def __len__(self):
        return len(self.keys)

    def __getitem__(self, idx):
        key = self.keys[idx]
        g = self._f()[key]
        z = np.asarray(g["elements"][:]).astype(np.int64)
        fock = restore_orca_diffuse_order(reinflate_symmetric(np.asarray(g["fock"][:])), z)
        attrs = getattr(g, "attrs", {})
        return {"z": z, "pos": np.asarray(g["coords"][:], dtype=np.float32), "fock": fock.astype(np.float32),
                "charge": int(float(attrs.get("charge", 0))), "spin": int(float(attrs.get("spin", 0))), "name": key}

    def close(self):
        if self._file is not None and hasattr(self._file, "close"):
            self._file.close()
        self._file = None
