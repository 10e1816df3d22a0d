"""One-electron integrals over contracted Gaussian shells, in this package's orbital order.

Overlap S, kinetic energy T and nuclear attraction V for real solid-harmonic Gaussian shells
(l <= 4), with the McMurchie-Davidson scheme (L. E. McMurchie and E. R. Davidson, J. Comput.
Phys. 26, 218 (1978); T. Helgaker, P. Jorgensen, J. Olsen, "Molecular Electronic-Structure
Theory", ch. 9): Hermite expansion coefficients E_t^{ij} per axis, overlap from E_0, kinetic
energy from overlaps of shifted angular momenta, nuclear attraction from Hermite Coulomb
integrals R_tuv built on the Boys function F_n(T) = 1F1(n + 1/2; n + 3/2; -T) / (2n + 1).

Orbital order and phases are those of the label layout (e3nn's real harmonics: inside a shell
m = -l..l, for l = 1 the order (y, z, x)); the solid-harmonic coefficients come from fitting the
package's own ``core.sph.real_sph_harm`` (polar axis y in the model frame, i.e. physical z),
so a Fock matrix converted into this order pairs with these integrals.  Contracted functions
are normalised to unit self-overlap.

With them :func:`hf_energy` evaluates the energy functional of a Fock matrix,
E = 1/2 Tr[P (H + F)] + E_nn with H = T + V, which is the total energy when F is a
Hartree-Fock Fock matrix (for a Kohn-Sham matrix the exchange-correlation correction, which
needs an XC grid, is not included).  Reference counterpart: ``fock_utils/get_energy_from_fock.py``
(PySCF core Hamiltonian and XC energy).
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
from scipy.special import hyp1f1

BOHR_PER_ANGSTROM = 1.0 / 0.52917721092
_L_OF = {"S": 0, "P": 1, "D": 2, "F": 3, "G": 4}


# ------------------------------------------------------------------ basis input
def parse_gaussian94(text):
    """Basis sets in the Gaussian94 text format -> {Z: [(l, exponents, coefficients), ...]}.

    Element blocks start with ``<symbol> 0`` and end with ``****``; shell lines are
    ``<type> <n_primitives> <scale>`` followed by ``exponent coefficient`` lines (``SP``
    shells carry two coefficient columns and become an s and a p shell).  Fortran ``D``
    exponents are accepted."""
    from ..data.readers import SYMBOL_TO_Z

    out = {}
    z = None
    lines = [ln.strip() for ln in text.splitlines()]
    i = 0
    while i < len(lines):
        ln = lines[i]
        if not ln or ln.startswith("!") or ln == "****":
            if ln == "****":
                z = None
            i += 1
            continue
        parts = ln.split()
        if z is None:
            z = SYMBOL_TO_Z[parts[0].capitalize()]
            out.setdefault(z, [])
            i += 1
            continue
        kind, n = parts[0].upper(), int(parts[1])
        rows = [[float(v.replace("D", "E").replace("d", "e")) for v in lines[i + 1 + k].split()] for k in range(n)]
        rows = np.array(rows)
        if kind == "SP":
            out[z].append((0, rows[:, 0], rows[:, 1]))
            out[z].append((1, rows[:, 0], rows[:, 2]))
        else:
            out[z].append((_L_OF[kind], rows[:, 0], rows[:, 1]))
        i += 1 + n
    return out


# ------------------------------------------------------------------ angular parts
def _cart_components(l):
    return [(a, b, l - a - b) for a in range(l, -1, -1) for b in range(l - a, -1, -1)]


@lru_cache(maxsize=None)
def solid_harmonic_coefficients(l):
    """C [2l+1, n_cart]: r^l Y_lm(r^) = sum_k C[m, k] x^a y^b z^c over the Cartesian components
    k = (a, b, c) (physical coordinates), Y the package's real harmonics."""
    from ..core.sph import real_sph_harm

    rng = np.random.default_rng(17 + l)
    pts = rng.normal(size=(6 * (l + 1) ** 2 + 20, 3)) * rng.uniform(0.5, 2.0, size=(1, 1))
    r = np.linalg.norm(pts, axis=1)
    model = pts[:, [1, 2, 0]] / r[:, None]  # model frame (x, y, z) = physical (y, z, x)
    Y = real_sph_harm(l, model) * r[:, None] ** l
    comps = _cart_components(l)
    M = np.stack([pts[:, 0] ** a * pts[:, 1] ** b * pts[:, 2] ** c for a, b, c in comps], axis=1)
    C = np.linalg.lstsq(M, Y, rcond=None)[0].T
    C[np.abs(C) < 1e-12] = 0.0
    return C


# ------------------------------------------------------------------ Hermite expansions
def _hermite_E(i, j, XAB, a, b):
    """E[i', j', t] for i' <= i, j' <= j along one axis; arrays over primitive pairs."""
    p = a + b
    mu = a * b / p
    XPA = -b / p * XAB
    XPB = a / p * XAB
    E = np.zeros((i + 1, j + 1, i + j + 2) + np.shape(a))
    E[0, 0, 0] = np.exp(-mu * XAB * XAB)
    for ii in range(i + 1):
        for jj in range(j + 1):
            if ii == 0 and jj == 0:
                continue
            for t in range(ii + jj + 1):
                if ii > 0:
                    v = XPA * E[ii - 1, jj, t] + (t + 1) * E[ii - 1, jj, t + 1]
                    if t > 0:
                        v = v + E[ii - 1, jj, t - 1] / (2 * p)
                else:
                    v = XPB * E[ii, jj - 1, t] + (t + 1) * E[ii, jj - 1, t + 1]
                    if t > 0:
                        v = v + E[ii, jj - 1, t - 1] / (2 * p)
                E[ii, jj, t] = v
    return E


def boys(n, T):
    """F_n(T) = integral_0^1 t^(2n) exp(-T t^2) dt."""
    return hyp1f1(n + 0.5, n + 1.5, -np.asarray(T, dtype=np.float64)) / (2 * n + 1)


def _hermite_R(L, p, PC):
    """R[t, u, v] (t + u + v <= L) of the Hermite Coulomb integrals, arrays [..., n_nuclei]."""
    X, Y, Z = PC[..., 0], PC[..., 1], PC[..., 2]
    T = p * (X * X + Y * Y + Z * Z)
    Rn = {}
    for n in range(L + 1):
        Rn[(n, 0, 0, 0)] = (-2 * p) ** n * boys(n, T)
    for tot in range(1, L + 1):
        for n in range(L - tot + 1):
            for t in range(tot + 1):
                for u in range(tot - t + 1):
                    v = tot - t - u
                    if t > 0:
                        val = X * Rn[(n + 1, t - 1, u, v)]
                        if t > 1:
                            val = val + (t - 1) * Rn[(n + 1, t - 2, u, v)]
                    elif u > 0:
                        val = Y * Rn[(n + 1, t, u - 1, v)]
                        if u > 1:
                            val = val + (u - 1) * Rn[(n + 1, t, u - 2, v)]
                    else:
                        val = Z * Rn[(n + 1, t, u, v - 1)]
                        if v > 1:
                            val = val + (v - 1) * Rn[(n + 1, t, u, v - 2)]
                    Rn[(n, t, u, v)] = val
    return {(t, u, v): Rn[(0, t, u, v)] for (n, t, u, v) in Rn if n == 0}


# ------------------------------------------------------------------ integrals
def _shells(z, pos_bohr, basis):
    """[(l, exponents, normalised primitive coefficients, centre)] in orbital order."""
    out = []
    for a, A in zip(z, pos_bohr):
        for l, exps, coefs in basis[int(a)]:
            exps = np.asarray(exps, dtype=np.float64)
            # primitive normalisation of the radial part up to a factor common to the shell
            # (the contracted functions are renormalised at the end)
            nrm = (2 * exps / math.pi) ** 0.75 * (4 * exps) ** (l / 2)
            out.append((l, exps, np.asarray(coefs, dtype=np.float64) * nrm, np.asarray(A, dtype=np.float64)))
    return out


def one_electron_integrals(z, pos, basis, units="angstrom"):
    """(S, T, V) [n_orb, n_orb] for atoms ``z`` at ``pos`` with ``basis`` = {Z: [(l, exponents,
    coefficients)]} (the shell order of each element is the orbital order); V includes every
    nucleus of charge Z."""
    z = np.asarray(z)
    pos = np.asarray(pos, dtype=np.float64) * (BOHR_PER_ANGSTROM if units == "angstrom" else 1.0)
    shells = _shells(z, pos, basis)
    sizes = [2 * l + 1 for l, *_ in shells]
    offs = np.concatenate([[0], np.cumsum(sizes)])
    n = int(offs[-1])
    S, T, V = np.zeros((n, n)), np.zeros((n, n)), np.zeros((n, n))
    charges = z.astype(np.float64)
    for ia, (la, ea, ca, A) in enumerate(shells):
        for ib in range(ia, len(shells)):
            lb, eb, cb, B = shells[ib]
            s, t, v = _shell_pair(la, ea, ca, A, lb, eb, cb, B, pos, charges)
            Ca, Cb = solid_harmonic_coefficients(la), solid_harmonic_coefficients(lb)
            for M, blk in ((S, s), (T, t), (V, v)):
                b2 = Ca @ blk @ Cb.T
                M[offs[ia]:offs[ia + 1], offs[ib]:offs[ib + 1]] = b2
                M[offs[ib]:offs[ib + 1], offs[ia]:offs[ia + 1]] = b2.T
    d = 1.0 / np.sqrt(np.diag(S))
    return S * np.outer(d, d), T * np.outer(d, d), V * np.outer(d, d)


def _shell_pair(la, ea, ca, A, lb, eb, cb, B, nuclei, charges):
    """Cartesian blocks [n_cart(la), n_cart(lb)] of S, T, V for one contracted shell pair."""
    a = ea[:, None] * np.ones_like(eb)[None, :]
    b = np.ones_like(ea)[:, None] * eb[None, :]
    w = ca[:, None] * cb[None, :]
    p = a + b
    P = (a[..., None] * A + b[..., None] * B) / p[..., None]
    E = [_hermite_E(la, lb + 2, A[k] - B[k], a, b) for k in range(3)]  # lb + 2 for the kinetic terms
    PC = P[:, :, None, :] - nuclei[None, None, :, :]
    R = _hermite_R(la + lb, p[..., None], PC)
    ca_, cb_ = _cart_components(la), _cart_components(lb)
    S = np.zeros((len(ca_), len(cb_)))
    T = np.zeros_like(S)
    V = np.zeros_like(S)
    sq = np.sqrt(math.pi / p)

    def s1(k, i, j):  # 1-D overlap of powers i, j along axis k
        return E[k][i, j, 0] * sq if j >= 0 else 0.0

    def t1(k, i, j):  # 1-D kinetic energy -1/2 d^2/dx^2 acting on the j side
        v = b * (2 * j + 1) * s1(k, i, j) - 2 * b * b * s1(k, i, j + 2)
        if j >= 2:
            v = v - 0.5 * j * (j - 1) * s1(k, i, j - 2)
        return v

    for x, (i1, j1, k1) in enumerate(ca_):
        for y, (i2, j2, k2) in enumerate(cb_):
            sx, sy, sz = s1(0, i1, i2), s1(1, j1, j2), s1(2, k1, k2)
            S[x, y] = np.sum(w * sx * sy * sz)
            T[x, y] = np.sum(w * (t1(0, i1, i2) * sy * sz + sx * t1(1, j1, j2) * sz + sx * sy * t1(2, k1, k2)))
            acc = 0.0
            for t in range(i1 + i2 + 1):
                Et = E[0][i1, i2, t]
                for u in range(j1 + j2 + 1):
                    Eu = E[1][j1, j2, u]
                    for vv in range(k1 + k2 + 1):
                        acc = acc + (Et * Eu * E[2][k1, k2, vv])[..., None] * R[(t, u, vv)]
            V[x, y] = -np.sum(w[..., None] * (2 * math.pi / p)[..., None] * acc * charges)
    return S, T, V


def nuclear_repulsion(z, pos, units="angstrom"):
    pos = np.asarray(pos, dtype=np.float64) * (BOHR_PER_ANGSTROM if units == "angstrom" else 1.0)
    z = np.asarray(z, dtype=np.float64)
    e = 0.0
    for i in range(len(z)):
        for j in range(i):
            e += z[i] * z[j] / np.linalg.norm(pos[i] - pos[j])
    return float(e)


def hf_energy(F, z, pos, basis, n_electrons=None, units="angstrom", tol=1e-6):
    """Energy functional of a closed-shell Fock matrix ``F`` (this package's orbital order):
    the density P of its lowest n/2 orbitals (generalised eigenproblem with the computed
    overlap), E = 1/2 Tr[P (H + F)] + E_nn with H = T + V.  Returns a dict with the energy and
    its parts (Hartree)."""
    from .electronic import closed_shell_density, n_electrons as count, orbitals

    S, T, V = one_electron_integrals(z, pos, basis, units)
    ne = count(z) if n_electrons is None else n_electrons
    F = 0.5 * (np.asarray(F, dtype=np.float64) + np.asarray(F, dtype=np.float64).T)
    e, C = orbitals(F, S, tol)
    P = closed_shell_density(C, ne)
    H = T + V
    e_el = 0.5 * float(np.sum(P * (H + F)))
    e_nn = nuclear_repulsion(z, pos, units)
    return {"total": e_el + e_nn, "electronic": e_el, "nuclear_repulsion": e_nn,
            "one_electron": float(np.sum(P * H)), "orbital_energies": e, "density": P, "overlap": S}


# ------------------------------------------------------------------ orbitals on a grid, files
def ao_values(points, z, pos, basis, units="angstrom"):
    """Values [n_points, n_orb] of the contracted orbitals (normalised as in
    :func:`one_electron_integrals`) at ``points`` (same units as ``pos``)."""
    f = BOHR_PER_ANGSTROM if units == "angstrom" else 1.0
    pts = np.asarray(points, dtype=np.float64) * f
    shells = _shells(np.asarray(z), np.asarray(pos, dtype=np.float64) * f, basis)
    cols = []
    for l, exps, coefs, A in shells:
        d = pts - A
        r2 = np.sum(d * d, axis=1)
        radial = np.exp(-r2[:, None] * exps[None, :]) @ coefs
        cart = np.stack([d[:, 0] ** a * d[:, 1] ** b * d[:, 2] ** c for a, b, c in _cart_components(l)], axis=1)
        cols.append((cart @ solid_harmonic_coefficients(l).T) * radial[:, None])
    vals = np.concatenate(cols, axis=1)
    # the normalisation of the integrals: divide by the norms of the unnormalised functions
    return vals / _raw_norms(z, pos, basis, units)[None, :]


def _raw_norms(z, pos, basis, units):
    f = BOHR_PER_ANGSTROM if units == "angstrom" else 1.0
    shells = _shells(np.asarray(z), np.asarray(pos, dtype=np.float64) * f, basis)
    out = []
    for l, e, c, A in shells:
        s, _, _ = _shell_pair(l, e, c, A, l, e, c, A, A[None, :], np.zeros(1))
        C = solid_harmonic_coefficients(l)
        out.append(np.sqrt(np.diag(C @ s @ C.T)))
    return np.concatenate(out)


def write_density_cube(path, z, pos, P, basis, spacing=0.4, margin=3.0):
    """Electron density rho(r) = sum_ij P_ij phi_i(r) phi_j(r) on a box around the molecule
    (``spacing`` and ``margin`` in Angstrom) as a Gaussian cube file (bohr units inside)."""
    pos = np.asarray(pos, dtype=np.float64)
    lo = pos.min(axis=0) - margin
    n = np.ceil((pos.max(axis=0) + margin - lo) / spacing).astype(int)
    axes = [lo[k] + spacing * np.arange(n[k]) for k in range(3)]
    X, Y, Z = np.meshgrid(*axes, indexing="ij")
    pts = np.stack([X.ravel(), Y.ravel(), Z.ravel()], axis=1)
    rho = np.empty(len(pts))
    for s0 in range(0, len(pts), 20000):
        a = ao_values(pts[s0:s0 + 20000], z, pos, basis)
        rho[s0:s0 + 20000] = np.einsum("pi,ij,pj->p", a, P, a)
    rho = rho.reshape(tuple(n))  # electrons per bohr^3 (the orbitals are functions of bohr coordinates)
    b = BOHR_PER_ANGSTROM
    with open(path, "w") as fh:
        fh.write("electron density\nwritten by maloq_b200\n")
        fh.write(f"{len(z):5d} {lo[0] * b:12.6f} {lo[1] * b:12.6f} {lo[2] * b:12.6f}\n")
        for k in range(3):
            v = [0.0, 0.0, 0.0]
            v[k] = spacing * b
            fh.write(f"{n[k]:5d} {v[0]:12.6f} {v[1]:12.6f} {v[2]:12.6f}\n")
        for zz, p in zip(z, pos):
            fh.write(f"{int(zz):5d} {float(zz):12.6f} {p[0] * b:12.6f} {p[1] * b:12.6f} {p[2] * b:12.6f}\n")
        flat = rho.reshape(n[0] * n[1], n[2])
        for row in flat:
            for s0 in range(0, len(row), 6):
                fh.write(" ".join(f"{v:13.5e}" for v in row[s0:s0 + 6]) + "\n")
    return path


def write_xyz(path, z, pos, comment="written by maloq_b200"):
    from ..data.readers import SYMBOL_TO_Z

    sym = {v: k for k, v in SYMBOL_TO_Z.items()}
    with open(path, "w") as fh:
        fh.write(f"{len(z)}\n{comment}\n")
        for zz, p in zip(z, np.asarray(pos, dtype=np.float64)):
            fh.write(f"{sym[int(zz)]:2s} {p[0]:20.10f} {p[1]:20.10f} {p[2]:20.10f}\n")
    return path


# ------------------------------------------------------------------ command line
def main(argv=None):
    """``python -m maloq_b200.eval.integrals STRUCTURE.xyz BASIS.g94 FOCK.npy [--cube rho.cube]``:
    the Hartree-Fock energy functional of a closed-shell Fock matrix (this package's orbital
    order) and optionally its electron-density cube (reference ``get_energy_from_fock.py``)."""
    import argparse

    from ..data.readers import SYMBOL_TO_Z

    ap = argparse.ArgumentParser(description="energy functional and density of a Fock matrix")
    ap.add_argument("xyz")
    ap.add_argument("basis")
    ap.add_argument("fock")
    ap.add_argument("--charge", type=int, default=0)
    ap.add_argument("--cube", default=None)
    ap.add_argument("--spacing", type=float, default=0.4)
    args = ap.parse_args(argv)
    with open(args.xyz) as fh:
        lines = fh.read().splitlines()
    n = int(lines[0].split()[0])
    z, pos = [], []
    for ln in lines[2:2 + n]:
        p = ln.split()
        z.append(SYMBOL_TO_Z[p[0].capitalize()])
        pos.append([float(v) for v in p[1:4]])
    with open(args.basis) as fh:
        basis = parse_gaussian94(fh.read())
    F = np.load(args.fock)
    res = hf_energy(F, z, np.array(pos), basis, n_electrons=int(sum(z)) - args.charge)
    print(f"E = {res['total']:.10f} Eh  (electronic {res['electronic']:.10f}, nuclear repulsion "
          f"{res['nuclear_repulsion']:.10f})")
    if args.cube:
        write_density_cube(args.cube, z, np.array(pos), res["density"], basis, spacing=args.spacing)
        print(f"density cube -> {args.cube}")
    return res


if __name__ == "__main__":
    main()
