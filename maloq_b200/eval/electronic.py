"""Orbital energies, densities and energies from a Fock/Kohn-Sham matrix.

The generalised eigenproblem F C = S C e is solved by canonical orthogonalisation
(Löwdin 1970): S = U s U^T, directions with s <= ``tol`` are dropped (near-linear
dependencies of diffuse basis sets), X = U_kept s_kept^{-1/2}, then F' = X^T F X is
diagonalised and C = X C'.  Closed shell: P = 2 C_occ C_occ^T.  Reference behaviour:
``fock_utils/get_energy_from_fock.py:82-123`` (same tolerance default, 0.1).  Total DFT
energies need the one-electron integrals and XC grids of PySCF (``total_energy``), which is
optional; everything else here is numpy/scipy.
"""

from __future__ import annotations

import numpy as np


def orthogonalizer(S, tol=1e-1):
    """X [n, r] with X^T S X = 1 on the kept subspace (overlap eigenvalues > tol)."""
    s, U = np.linalg.eigh(np.asarray(S, dtype=np.float64))
    keep = s > tol
    return U[:, keep] / np.sqrt(s[keep])


def orbitals(F, S=None, tol=1e-1):
    """Orbital energies (ascending) and coefficients of F (generalised with S if given)."""
    F = 0.5 * (np.asarray(F, dtype=np.float64) + np.asarray(F, dtype=np.float64).T)
    if S is None:
        return np.linalg.eigh(F)
    X = orthogonalizer(S, tol)
    e, Cp = np.linalg.eigh(X.T @ F @ X)
    return e, X @ Cp


def n_electrons(z, charge=0):
    return int(np.sum(np.asarray(z))) - int(charge)


def closed_shell_density(C, n_elec):
    nocc = n_elec // 2
    Co = C[:, :nocc]
    return 2.0 * Co @ Co.T


def summary(F, S=None, n_elec=None, tol=1e-1):
    """Orbital energies, HOMO/LUMO, gap and band energy (2 * sum of occupied orbital
    energies, closed shell).  Occupation-dependent entries are None when ``n_elec`` is not
    given or needs more orbitals than the basis has."""
    e, C = orbitals(F, S, tol)
    out = {"eigenvalues": e, "homo": None, "lumo": None, "gap": None, "band_energy": None, "density": None}
    if n_elec is not None:
        nocc = n_elec // 2
        if 0 < nocc < len(e):
            out.update(homo=float(e[nocc - 1]), lumo=float(e[nocc]), gap=float(e[nocc] - e[nocc - 1]),
                       band_energy=float(2.0 * e[:nocc].sum()), density=closed_shell_density(C, n_elec))
    return out


def total_energy(mol, F, S=None, xc="b3lyp", tol=1e-1):
    """Total DFT energy of the density built from F (needs PySCF; ``mol`` a pyscf Mole)."""
    try:
        from pyscf import dft  # noqa: F401
    except ImportError as e:  # pragma: no cover - pyscf is optional
        raise ImportError("total_energy needs PySCF, which is not installed") from e
    S = mol.intor("int1e_ovlp") if S is None else S
    e, C = orbitals(F, S, tol)
    P = closed_shell_density(C, mol.nelectron)
    mf = dft.RKS(mol)
    mf.xc = xc
    return float(mf.energy_tot(dm=P))
