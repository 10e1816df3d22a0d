"""One-electron integrals (McMurchie-Davidson) and the Hartree-Fock energy functional of a Fock
matrix, against published minimal-basis values and invariances."""
import math

import numpy as np
import pytest

from maloq_b200.eval import integrals as I

# STO-3G hydrogen (zeta = 1.24): a published basis-set table
H_STO3G = {1: [(0, [3.42525091, 0.62391373, 0.16885540], [0.15432897, 0.53532814, 0.44463454])]}


def test_h2_sto3g_integrals_and_hf_energy():
    """H2 at R = 1.4 bohr in STO-3G: the overlap, kinetic, nuclear-attraction and core
    Hamiltonian matrix elements and the Hartree-Fock total energy -1.1167 Eh tabulated by
    Szabo and Ostlund ("Modern Quantum Chemistry", section 3.5.2)."""
    z = [1, 1]
    pos = np.array([[0.0, 0.0, 0.0], [0.0, 0.0, 1.4]])
    S, T, V = I.one_electron_integrals(z, pos, H_STO3G, units="bohr")
    assert abs(S[0, 1] - 0.6593) < 1e-4
    assert abs(T[0, 0] - 0.7600) < 1e-4 and abs(T[0, 1] - 0.2365) < 1e-4
    H = T + V
    assert abs(H[0, 0] + 1.1204) < 1e-4 and abs(H[0, 1] + 0.9584) < 1e-4
    # the converged closed-shell Fock matrix needs the (ss|ss) repulsion integrals; with one
    # orbital of each symmetry the SCF density is the sigma_g orbital's
    eri = _ss_eri(pos, *H_STO3G[1][0][1:])
    c = np.array([1.0, 1.0]) / math.sqrt(2 * (1 + S[0, 1]))
    P = 2 * np.outer(c, c)
    G = np.einsum("ls,mnsl->mn", P, eri) - 0.5 * np.einsum("ls,mlsn->mn", P, eri)
    F = H + G
    res = I.hf_energy(F, z, pos, H_STO3G, units="bohr")
    assert abs(res["total"] + 1.1167) < 1e-4
    assert abs(res["nuclear_repulsion"] - 1 / 1.4) < 1e-12


def _ss_eri(pos, exps, coefs):
    """(ab|cd) over normalised s-type contractions on the given centres (closed form with F0)."""
    exps, coefs = np.asarray(exps), np.asarray(coefs)
    nrm = coefs * (2 * exps / math.pi) ** 0.75
    n = len(pos)
    out = np.zeros((n, n, n, n))
    for a in range(n):
        for b in range(n):
            for c in range(n):
                for d in range(n):
                    acc = 0.0
                    for i, ai in enumerate(exps):
                        for j, bj in enumerate(exps):
                            p = ai + bj
                            Pp = (ai * pos[a] + bj * pos[b]) / p
                            kab = math.exp(-ai * bj / p * np.sum((pos[a] - pos[b]) ** 2))
                            for k, ck in enumerate(exps):
                                for m, dm in enumerate(exps):
                                    q = ck + dm
                                    Q = (ck * pos[c] + dm * pos[d]) / q
                                    kcd = math.exp(-ck * dm / q * np.sum((pos[c] - pos[d]) ** 2))
                                    Tq = p * q / (p + q) * np.sum((Pp - Q) ** 2)
                                    acc += nrm[i] * nrm[j] * nrm[k] * nrm[m] * 2 * math.pi ** 2.5 / (
                                        p * q * math.sqrt(p + q)) * kab * kcd * float(I.boys(0, Tq))
                    out[a, b, c, d] = acc
    return out


def _toy_basis():
    """Made-up shells up to f (exponents / coefficients arbitrary but positive)."""
    return {8: [(0, [5.0, 1.1], [0.4, 0.7]), (1, [3.0, 0.6], [0.5, 0.6]), (2, [1.2], [1.0]), (3, [0.9], [1.0])],
            1: [(0, [2.0, 0.4], [0.5, 0.6]), (1, [0.8], [1.0])]}


def _rotation(seed):
    q = np.random.default_rng(seed).normal(size=4)
    a, b, c, d = q / np.linalg.norm(q)
    return np.array([[a * a + b * b - c * c - d * d, 2 * (b * c - a * d), 2 * (b * d + a * c)],
                     [2 * (b * c + a * d), a * a - b * b + c * c - d * d, 2 * (c * d - a * b)],
                     [2 * (b * d - a * c), 2 * (c * d + a * b), a * a - b * b - c * c + d * d]])


def test_integrals_rotate_with_the_package_wigner_matrices():
    """Rotating the molecule by R changes every integral matrix to D S D^T with D the
    block-diagonal Wigner matrices of this package (the orbitals are its real harmonics, in the
    model frame); S has a unit diagonal and is positive definite."""
    from maloq_b200.core import sph

    z = [8, 1, 1]
    pos = np.array([[0.0, 0.1, 0.0], [0.76, -0.5, 0.1], [-0.7, -0.45, -0.2]])
    basis = _toy_basis()
    S, T, V = I.one_electron_integrals(z, pos, basis)
    assert np.allclose(np.diag(S), 1.0) and np.linalg.eigvalsh(S).min() > 0
    R = _rotation(3)
    S2, T2, V2 = I.one_electron_integrals(z, pos @ R.T, basis)
    perm = [1, 2, 0]  # physical -> model frame
    Rm = R[np.ix_(perm, perm)]
    blocks = []
    for a in z:
        for l, *_ in basis[a]:
            blocks.append(sph.wigner_D_from_matrix(l, Rm))
    n = sum(b.shape[0] for b in blocks)
    D = np.zeros((n, n))
    o = 0
    for b in blocks:
        D[o:o + len(b), o:o + len(b)] = b
        o += len(b)
    for M, M2 in ((S, S2), (T, T2), (V, V2)):
        assert np.allclose(D @ M @ D.T, M2, atol=1e-9)


def test_overlap_and_kinetic_energy_against_a_grid():
    """S and T of p, d and f shells on two centres against direct numerical integration of the
    contracted functions (built here from the solid-harmonic coefficients) on a product grid."""
    basis = {8: [(1, [1.3], [1.0]), (2, [0.9], [1.0]), (3, [0.7], [1.0])]}
    pos = np.array([[0.0, 0.0, 0.0], [0.3, -0.4, 0.5]])  # bohr
    S, T, _ = I.one_electron_integrals([8, 8], pos, basis, units="bohr")
    g = np.linspace(-6.5, 6.5, 105)
    h = g[1] - g[0]
    X, Y, Z = np.meshgrid(g, g, g, indexing="ij")

    def aos(center):
        x, y, zz = X - center[0], Y - center[1], Z - center[2]
        r2 = x * x + y * y + zz * zz
        out = []
        for l, (e,), _ in basis[8]:
            C = I.solid_harmonic_coefficients(l)
            cart = [x ** a * y ** b * zz ** c for a, b, c in I._cart_components(l)]
            for m in range(2 * l + 1):
                out.append(sum(C[m, k] * cart[k] for k in range(len(cart))) * np.exp(-e * r2))
        return out

    f = aos(pos[0]) + aos(pos[1])
    norms = [math.sqrt(np.sum(u * u) * h ** 3) for u in f]
    f = [u / s for u, s in zip(f, norms)]
    # kinetic energy 1/2 <grad f_i . grad f_j> with spectral derivatives (Parseval on the grid)
    k = 2 * np.pi * np.fft.fftfreq(len(g), d=h)
    KX, KY, KZ = np.meshgrid(k, k, k, indexing="ij")
    k2 = KX ** 2 + KY ** 2 + KZ ** 2
    for i, j in [(0, 15), (4, 20), (9, 22), (3, 3), (10, 28)]:
        s = np.sum(f[i] * f[j]) * h ** 3
        assert abs(s - S[i, j]) < 2e-4, (i, j, s, S[i, j])
        fi, fj = np.fft.fftn(f[i]), np.fft.fftn(f[j])
        t = 0.5 * np.real(np.sum(k2 * np.conj(fi) * fj)) * h ** 3 / f[i].size
        assert abs(t - T[i, j]) < 1e-3, (i, j, t, T[i, j])


def test_nuclear_attraction_far_nucleus_and_h_like_atom():
    """V from a distant point charge tends to -Z S / |R| within a d or f shell; the STO-3G
    hydrogen 1s (zeta = 1.24) in the field of its own nucleus gives the tabulated -1.2266."""
    basis = {8: [(2, [1.1, 0.4], [0.6, 0.5]), (3, [0.8], [1.0])], 1: [(0, [1.0], [1.0])]}
    pos = np.array([[0.0, 0.0, 0.0], [0.2, -0.3, 0.1], [400.0, 300.0, -200.0]])  # bohr; far H nucleus
    S, _, V = I.one_electron_integrals([8, 8, 1], pos, basis, units="bohr")
    n = 24  # the two O atoms' d + f functions
    S0, _, V0 = I.one_electron_integrals([8, 8], pos[:2], basis, units="bohr")
    Vfar = V[:n, :n] - V0  # the far H nucleus alone (V0 holds the two O nuclei)
    # same-shell blocks have no dipole moment (parity), so the next correction falls off as d^-3
    for a, b, atom in ((0, 5, 0), (5, 12, 0), (12, 17, 1), (17, 24, 1)):
        d = np.linalg.norm(pos[2] - pos[atom])
        assert np.allclose(Vfar[a:b, a:b], -1.0 * S0[a:b, a:b] / d, rtol=0, atol=5e-8)
    _, _, Vh = I.one_electron_integrals([1], np.zeros((1, 3)), {1: [(0, [3.42525091, 0.62391373, 0.16885540],
                                                                    [0.15432897, 0.53532814, 0.44463454])]},
                                       units="bohr")
    assert abs(Vh[0, 0] + 1.2266) < 1e-4  # V^1_11 of Szabo and Ostlund (zeta = 1.24)


def test_gaussian94_parser():
    text = """! comment
H     0
S   3   1.00
      3.42525091             0.15432897
      0.62391373             0.53532814
      0.16885540             0.44463454
****
O     0
S   1   1.00
    130.70932D+00           1.0
SP   2   1.00
      5.0331513             -0.09996723            0.15591627
      1.1695961              0.39951283            0.60768372
****
"""
    b = I.parse_gaussian94(text)
    assert [l for l, *_ in b[1]] == [0] and np.allclose(b[1][0][1], H_STO3G[1][0][1])
    assert [l for l, *_ in b[8]] == [0, 0, 1]
    assert np.isclose(b[8][0][1][0], 130.70932)
    assert np.allclose(b[8][2][2], [0.15591627, 0.60768372])


def test_orbitals_on_a_grid_density_cube_and_xyz(tmp_path):
    """Orbital values reproduce the overlap matrix by quadrature; the density of P integrates to
    Tr[P S] electrons; the cube and xyz files have the standard layouts."""
    basis = _toy_basis()
    z = [8, 1, 1]
    pos = np.array([[0.0, 0.1, 0.0], [0.76, -0.5, 0.1], [-0.7, -0.45, -0.2]])  # Angstrom
    S, _, _ = I.one_electron_integrals(z, pos, basis)
    g = np.linspace(-5.0, 5.0, 81)  # Angstrom
    h = (g[1] - g[0]) * I.BOHR_PER_ANGSTROM
    X, Y, Z = np.meshgrid(g, g, g, indexing="ij")
    a = I.ao_values(np.stack([X.ravel(), Y.ravel(), Z.ravel()], 1), z, pos, basis)
    Sq = a.T @ a * h ** 3
    assert np.abs(Sq - S).max() < 2e-3
    rng = np.random.default_rng(0)
    C = rng.normal(size=(S.shape[0], 5))
    P = C @ C.T
    path = I.write_density_cube(str(tmp_path / "rho.cube"), z, pos, P, basis, spacing=0.15, margin=4.0)
    lines = open(path).read().splitlines()
    n = [int(lines[3 + k].split()[0]) for k in range(3)]
    vals = np.array([float(v) for ln in lines[6 + len(z):] for v in ln.split()])
    assert vals.size == n[0] * n[1] * n[2]
    dv = (0.15 * I.BOHR_PER_ANGSTROM) ** 3
    assert abs(vals.sum() * dv - np.sum(P * S)) < 2e-2 * np.sum(P * S)
    xyz = open(I.write_xyz(str(tmp_path / "m.xyz"), z, pos)).read().splitlines()
    assert xyz[0] == "3" and xyz[2].split()[0] == "O" and float(xyz[3].split()[1]) == 0.76


def test_energy_command_line(tmp_path, capsys):
    """The energy/cube command on H2 in STO-3G with its SCF Fock matrix."""
    pos = np.array([[0.0, 0.0, 0.0], [0.0, 0.0, 1.4]]) / I.BOHR_PER_ANGSTROM
    S, T, V = I.one_electron_integrals([1, 1], pos, H_STO3G)
    eri = _ss_eri(pos * I.BOHR_PER_ANGSTROM, *H_STO3G[1][0][1:])
    c = np.array([1.0, 1.0]) / math.sqrt(2 * (1 + S[0, 1]))
    P = 2 * np.outer(c, c)
    F = T + V + np.einsum("ls,mnsl->mn", P, eri) - 0.5 * np.einsum("ls,mlsn->mn", P, eri)
    np.save(tmp_path / "F.npy", F)
    I.write_xyz(str(tmp_path / "h2.xyz"), [1, 1], pos)
    (tmp_path / "b.g94").write_text("H 0\nS 3 1.00\n 3.42525091 0.15432897\n 0.62391373 0.53532814\n"
                                    " 0.16885540 0.44463454\n****\n")
    res = I.main([str(tmp_path / "h2.xyz"), str(tmp_path / "b.g94"), str(tmp_path / "F.npy"), "--cube",
                  str(tmp_path / "h2.cube"), "--spacing", "0.3"])
    assert abs(res["total"] + 1.1167) < 1e-4 and "E = -1.116" in capsys.readouterr().out
    assert (tmp_path / "h2.cube").exists()
