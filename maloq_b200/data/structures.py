"""Synthetic molecules and materials with the shapes of the benchmark configurations.

No datasets are available offline, so structures are generated:

* :func:`random_small_molecule` - 3-9 atoms from {H,C,N,O} uniform in a 4 A cube,
  rejection-sampled to a 0.9 A minimum pair distance;
* :func:`random_druglike_molecule` - a random bonded heavy-atom tree with ring closures
  (1.0-1.6 A bonds), hydrogens attached, relaxed by gradient steps on harmonic bonds plus
  a soft pair repulsion;
* :func:`amorphous_sio2` - Si:O = 1:2 at a target density with a minimum distance, in an
  orthorhombic periodic box;
* :func:`si_slab_with_oxide` - diamond-lattice Si slab, a Hf/O-substituted oxide layer
  and thermal displacements.
"""

from __future__ import annotations

import numpy as np

from .basis_sets import Br, C, Cl, F, H, Hf, N, O, P, S, Si

MASS = {H: 1.008, C: 12.011, N: 14.007, O: 15.999, F: 18.998, P: 30.974, S: 32.06, Cl: 35.45, Br: 79.904,
        Si: 28.086, Hf: 178.49}


class Structure:
    """Atomic numbers, positions [n, 3] (A), optional orthorhombic cell [3], charge, spin."""

    def __init__(self, z, pos, cell=None, charge=0, spin=1):
        self.z = np.asarray(z, dtype=np.int64)
        self.pos = np.asarray(pos, dtype=np.float64)
        self.cell = None if cell is None else np.asarray(cell, dtype=np.float64)
        self.charge, self.spin = int(charge), int(spin)

    def __len__(self):
        return len(self.z)


def random_small_molecule(rng, n_min=3, n_max=9, elements=(H, C, N, O), box=4.0, dmin=0.9):
    n = int(rng.integers(n_min, n_max + 1))
    pos = []
    while len(pos) < n:
        p = rng.uniform(0, box, size=3)
        if all(np.linalg.norm(p - q) >= dmin for q in pos):
            pos.append(p)
    z = rng.choice(elements, size=n)
    return Structure(z, np.array(pos))


def _relax(pos, bonds, steps=60, lr=0.05, r0=None, rep_cut=2.0):
    """Gradient steps on sum_bonds (|d|-r0)^2 + sum_nonbonded max(0, rep_cut-|d|)^2."""
    n = len(pos)
    bonded = np.zeros((n, n), dtype=bool)
    if len(bonds):
        bonded[bonds[:, 0], bonds[:, 1]] = bonded[bonds[:, 1], bonds[:, 0]] = True
    np.fill_diagonal(bonded, True)
    for _ in range(steps):
        d = pos[:, None, :] - pos[None, :, :]
        r = np.linalg.norm(d, axis=-1) + 1e-9
        grad = np.zeros_like(pos)
        rep = np.where(~bonded & (r < rep_cut), rep_cut - r, 0.0)
        grad -= 2 * ((rep / r)[..., None] * d).sum(axis=1)
        if len(bonds):
            i, j = bonds[:, 0], bonds[:, 1]
            dv = pos[i] - pos[j]
            rb = np.linalg.norm(dv, axis=-1) + 1e-9
            f = 2 * ((rb - r0) / rb)[:, None] * dv
            np.add.at(grad, i, f)
            np.add.at(grad, j, -f)
        pos = pos - lr * grad
    return pos


def random_druglike_molecule(rng, n_min=30, n_max=50, heavy=(C, N, O, F, S, Cl),
                             freq=None):
    """Random bonded chain/ring molecule; element frequencies H 45%, C 35%, N 8%, O 8%, rest even."""
    n = int(rng.integers(n_min, n_max + 1))
    if freq is None:
        rest = [e for e in heavy if e not in (C, N, O)]
        freq = {H: 0.45, C: 0.35, N: 0.08, O: 0.08}
        for e in rest:
            freq[e] = 0.04 / len(rest)
    els = list(freq)
    p = np.array([freq[e] for e in els])
    z = rng.choice(els, size=n, p=p / p.sum())
    heavy_idx = [i for i in range(n) if z[i] != H]
    if not heavy_idx:
        z[0] = C
        heavy_idx = [0]
    h_idx = [i for i in range(n) if z[i] == H]
    pos = np.zeros((n, 3))
    bonds = []
    r0 = []
    placed = [heavy_idx[0]]
    for i in heavy_idx[1:]:
        # attach to a recent heavy atom (chains) or a random one (branches)
        parent = placed[-1] if rng.random() < 0.7 else placed[int(rng.integers(len(placed)))]
        b = rng.uniform(1.2, 1.6)
        v = rng.normal(size=3)
        pos[i] = pos[parent] + b * v / np.linalg.norm(v)
        bonds.append((parent, i))
        r0.append(b)
        placed.append(i)
    # ring closures between heavy atoms 4-6 bonds apart
    for _ in range(max(1, len(heavy_idx) // 8)):
        if len(placed) < 7:
            break
        a = int(rng.integers(0, len(placed) - 6))
        k = int(rng.integers(4, 7))
        bonds.append((placed[a], placed[a + k]))
        r0.append(rng.uniform(1.3, 1.5))
    for i in h_idx:
        parent = heavy_idx[int(rng.integers(len(heavy_idx)))]
        b = rng.uniform(1.0, 1.1)
        v = rng.normal(size=3)
        pos[i] = pos[parent] + b * v / np.linalg.norm(v)
        bonds.append((parent, i))
        r0.append(b)
    pos = _relax(pos, np.array(bonds, dtype=np.int64), r0=np.array(r0))
    pos -= pos.mean(axis=0)
    return Structure(z, pos)


def random_large_molecule(rng, n_min=10, n_max=150):
    return random_druglike_molecule(rng, n_min, n_max, heavy=(C, N, O, F, P, S, Cl, Br))


def _poisson_fill(rng, n, cell, dmin, max_tries=200):
    """Random positions with a minimum (periodic) distance, using a cell grid."""
    cell = np.asarray(cell, dtype=np.float64)
    ncell = np.maximum((cell / dmin).astype(int), 1)
    h = cell / ncell
    grid = {}
    pos = np.zeros((n, 3))
    k = 0
    tries = 0
    while k < n:
        p = rng.uniform(0, 1, size=3) * cell
        c = tuple((p / h).astype(int) % ncell)
        ok = True
        for dx in (-1, 0, 1):
            for dy in (-1, 0, 1):
                for dz in (-1, 0, 1):
                    cc = ((c[0] + dx) % ncell[0], (c[1] + dy) % ncell[1], (c[2] + dz) % ncell[2])
                    for j in grid.get(cc, ()):
                        d = pos[j] - p
                        d -= cell * np.round(d / cell)
                        if d @ d < dmin * dmin:
                            ok = False
                            break
                    if not ok:
                        break
                if not ok:
                    break
        tries += 1
        if ok or tries > max_tries:
            grid.setdefault(c, []).append(k)
            pos[k] = p
            k += 1
            tries = 0
    return pos


def amorphous_sio2(rng, n_atoms=20000, density=2.2, dmin=1.5):
    """Si:O = 1:2 random amorphous-like supercell (orthorhombic, cubic box from density)."""
    n_si = n_atoms // 3
    z = np.array([Si] * n_si + [O] * (n_atoms - n_si))
    rng.shuffle(z)
    mass_g = sum(MASS[int(a)] for a in z) / 6.02214076e23
    vol_A3 = mass_g / density * 1e24
    a = vol_A3 ** (1 / 3)
    cell = np.array([a, a, a])
    pos = _poisson_fill(rng, n_atoms, cell, dmin)
    return Structure(z, pos, cell)


def si_slab_with_oxide(rng, n_atoms=1_000_000, a=5.43, oxide_nm=3.0, sub_frac=0.10, sigma=0.05):
    """Diamond Si slab of ~n_atoms; a top layer of ``oxide_nm`` has ``sub_frac`` of sites
    replaced by Hf/O; positions get Gaussian displacements of ``sigma`` A.  Periodic in x, y."""
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
                      [.25, .25, .25], [.25, .75, .75], [.75, .25, .75], [.75, .75, .25]])
    ncell = max(1, round((n_atoms / 8) ** (1 / 3)))
    nz = max(1, int(round(n_atoms / 8 / ncell / ncell)))
    ii, jj, kk = np.meshgrid(np.arange(ncell), np.arange(ncell), np.arange(nz), indexing="ij")
    origins = np.stack([ii, jj, kk], -1).reshape(-1, 1, 3)
    pos = ((origins + basis[None]) * a).reshape(-1, 3)
    z = np.full(len(pos), Si, dtype=np.int64)
    top = pos[:, 2].max()
    layer = pos[:, 2] > top - oxide_nm * 10
    sub = layer & (rng.random(len(pos)) < sub_frac)
    z[sub] = np.where(rng.random(int(sub.sum())) < 0.33, Hf, O)
    pos = pos + rng.normal(scale=sigma, size=pos.shape)
    cell = np.array([ncell * a, ncell * a, nz * a + 20.0])  # vacuum along z
    return Structure(z, pos, cell)


def tile_structure(st: Structure, tiling_dims) -> Structure:
    """Supercell of a periodic structure: ``tiling_dims`` = (n_a, n_b, n_c) copies along the
    (orthorhombic) cell axes.  Copies are ordered with the last axis fastest and each copy
    holds all atoms in their original order, so tiled atom t is original atom t % n (the
    order of ASE's ``atoms * dims``, which the reference uses, ``fock_targets_batched.py:1196``)."""
    if st.cell is None:
        raise ValueError("tiling needs a periodic structure (a cell)")
    dims = [int(d) for d in tiling_dims]
    if len(dims) != 3 or min(dims) < 1:
        raise ValueError(f"tiling_dims must be three positive integers, got {tiling_dims}")
    cell = np.asarray(st.cell, dtype=np.float64)
    shifts = np.array([(a, b, c) for a in range(dims[0]) for b in range(dims[1]) for c in range(dims[2])],
                      dtype=np.float64) * cell
    pos = (st.pos[None] + shifts[:, None]).reshape(-1, 3)
    return Structure(np.tile(st.z, len(shifts)), pos, cell * np.asarray(dims, dtype=np.float64), st.charge, st.spin)
