"""Dataset readers and orbital-order conventions.

* :class:`NablaDFTDatabase` - the nablaDFT Hamiltonian SQLite format (tables ``data``
  (id, Z, R, E, F, H, S, C as float32/int32 blobs), ``dataset_ids`` and ``metadata``), read
  with the standard-library ``sqlite3`` (reference ``dataset_utils/nablaDFT_dataset_utils.py``
  uses apsw for the same file).
* :func:`reorder_orbitals` - converts a matrix from a DFT code's orbital order to the
  e3nn real-harmonic order used by the labels (m = -l..l, y polar axis).  The per-code
  tables list each code's published ordering of p and d functions (kept identical to the
  reference's ``convention_dict`` because they describe the external programs' outputs).
* :func:`load_nabladft` - database rows -> graph samples with coupled-basis targets.
* CP2K periodic data: :func:`read_cp2k_csr` (binary or ASCII sparse dumps, symmetrised),
  :func:`read_periodic_xyz` (``Lattice=``/``Cell:`` headers), :func:`fermi_energy` and
  :func:`fermi_shift`, :func:`blocks_from_sparse` (atom-pair blocks without densifying) and
  :func:`load_cp2k`.
* ORCA output: :func:`read_orca_output` (coordinates, contracted basis, printed Fock
  matrices, total energy).
"""

from __future__ import annotations

import math
import os
import sqlite3

import numpy as np

BOHR_TO_ANGSTROM = 0.52917721092

# code -> shell letter -> (index permutation into e3nn order, signs)
CONVENTIONS = {
    "psi4": {"s": ([0], [1]), "p": ([2, 0, 1], [1, 1, 1]), "d": ([4, 2, 0, 1, 3], [1, 1, 1, 1, 1])},
    "orca": {"s": ([0], [1]), "p": ([2, 0, 1], [1, 1, 1]), "d": ([4, 2, 0, 1, 3], [1, 1, 1, 1, 1]),
             "f": ([6, 4, 2, 0, 1, 3, 5], [-1, 1, 1, 1, 1, 1, -1]),
             "g": ([8, 6, 4, 2, 0, 1, 3, 5, 7], [-1, -1, 1, 1, 1, 1, 1, -1, -1])},
    "pyscf": {"s": ([0], [1]), "p": ([1, 2, 0], [1, 1, 1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, 1, 1]),
              "f": ([0, 1, 2, 3, 4, 5, 6], [-1, 1, 1, 1, 1, 1, -1]),
              "g": ([0, 1, 2, 3, 4, 5, 6, 7, 8], [-1, -1, 1, 1, 1, 1, 1, -1, -1])},
    "aims": {"s": ([0], [1]), "p": ([0, 1, 2], [1, 1, -1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, -1, 1])},
    "e3nn": {"s": ([0], [1]), "p": ([0, 1, 2], [1, 1, 1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, 1, 1]),
             "f": ([0, 1, 2, 3, 4, 5, 6], [1] * 7)},
}
_L_LETTER = {0: "s", 1: "p", 2: "d", 3: "f", 4: "g"}


def reorder_indices(z, basis, convention="psi4"):
    """(index permutation, signs) taking a code-ordered matrix to e3nn order:
    ``H_e3nn = (H[idx][:, idx]) * sign[:, None] * sign[None, :]``."""
    conv = CONVENTIONS[convention]
    idx, sgn, off = [], [], 0
    for a in z:
        for l in basis[int(a)]:
            p, s = conv[_L_LETTER[l % 10]]
            idx += [off + i for i in p]
            sgn += list(s)
            off += 2 * (l % 10) + 1
    return np.asarray(idx, dtype=np.int64), np.asarray(sgn, dtype=np.float64)


def reorder_orbitals(H, z, basis, convention="psi4"):
    idx, sgn = reorder_indices(z, basis, convention)
    return H[..., idx, :][..., :, idx] * sgn[:, None] * sgn[None, :]


def reorder_orbitals_inverse(H, z, basis, convention="psi4"):
    """Inverse of :func:`reorder_orbitals`: an e3nn-ordered matrix back to the code's order."""
    idx, sgn = reorder_indices(z, basis, convention)
    out = np.empty_like(H)
    out[..., idx[:, None], idx[None, :]] = H * sgn[:, None] * sgn[None, :]
    return out


class NablaDFTDatabase:
    """Read-only access to a nablaDFT Hamiltonian database."""

    def __init__(self, path):
        self.path = path
        self.conn = sqlite3.connect(f"file:{path}?mode=ro", uri=True)

    def __len__(self):
        row = self.conn.execute("SELECT * FROM metadata WHERE id=0").fetchone()
        return int(row[-1])

    @staticmethod
    def _unpack(row):
        N = len(row[2]) // 12
        Z = np.frombuffer(row[1], dtype=np.int32).reshape(N).copy()
        R = np.frombuffer(row[2], dtype=np.float32).reshape(N, 3).copy()
        E = np.array([0.0 if row[3] is None else row[3]], dtype=np.float32)
        F = np.frombuffer(row[4], dtype=np.float32).reshape(N, 3).copy()
        n = int(math.isqrt(len(row[5]) // 4))
        H = np.frombuffer(row[5], dtype=np.float32).reshape(n, n).copy()
        S = np.frombuffer(row[6], dtype=np.float32).reshape(n, n).copy()
        C = np.frombuffer(row[7], dtype=np.float32).reshape(n, n).copy() if row[7] is not None else None
        return Z, R, E, F, H, S, C

    def __getitem__(self, idx):
        row = self.conn.execute("SELECT * FROM data WHERE id=?", (int(idx),)).fetchone()
        if row is None:
            raise IndexError(idx)
        return self._unpack(row)


def write_nabladft(path, molecules):
    """Write ``molecules`` = [(Z, R_bohr, E, F, H, S, C)] in the nablaDFT layout (used by tests
    and by tools that export synthetic data)."""
    conn = sqlite3.connect(path)
    conn.execute("CREATE TABLE IF NOT EXISTS data (id INTEGER NOT NULL PRIMARY KEY, Z BLOB, R BLOB, E FLOAT, "
                 "F BLOB, H BLOB, S BLOB, C BLOB)")
    conn.execute("CREATE TABLE IF NOT EXISTS dataset_ids (id INTEGER NOT NULL PRIMARY KEY, moses_id INT, "
                 "conformer_id INT)")
    conn.execute("CREATE TABLE IF NOT EXISTS metadata (id INTEGER PRIMARY KEY, N INTEGER)")
    for i, (Z, R, E, F, H, S, C) in enumerate(molecules):
        conn.execute("INSERT INTO data VALUES (?,?,?,?,?,?,?,?)",
                     (i, np.asarray(Z, np.int32).tobytes(), np.asarray(R, np.float32).tobytes(), float(E),
                      np.asarray(F, np.float32).tobytes(), np.asarray(H, np.float32).tobytes(),
                      np.asarray(S, np.float32).tobytes(), np.asarray(C, np.float32).tobytes()))
        conn.execute("INSERT INTO dataset_ids VALUES (?,?,?)", (i, i, 0))
    conn.execute("INSERT OR REPLACE INTO metadata VALUES (0, ?)", (len(molecules),))
    conn.commit()
    conn.close()


def load_nabladft(path, config, device="cpu", convention="psi4", indices=None):
    """Samples with coupled-basis targets from a nablaDFT database (def2-SVP basis)."""
    db = NablaDFTDatabase(path)
    n = len(db) if indices is None else None
    idx = list(range(min(n, config.get("num_structures", n)))) if indices is None else list(indices)

    def mols():
        for i in idx:
            Z, R, E, F, H, S, C = db[i]
            yield {"z": Z, "pos": R * BOHR_TO_ANGSTROM, "H": H.astype(np.float64), "S": S, "energy": float(E[0]),
                   "forces": F.astype(np.float64)}

    return molecules_to_samples(mols(), "def2_svp_nabla", config, device, convention=convention)


def load_qm7(path, config, device="cpu", indices=None):
    """The QM7 Hamiltonian ASE database (schnetpack rows: ``hamiltonian``, ``overlap``,
    ``energy``, ``forces`` in ORCA orbital order, def2-SVP; reference
    ``dataset_utils/get_loader.py:48-79``)."""
    from .asedb import ASEAtomsData

    db = ASEAtomsData(path)
    idx = list(range(min(len(db), config.get("num_structures") or len(db)))) if indices is None else list(indices)

    def mols():
        for i in idx:
            r = db[i]
            yield {"z": r["_atomic_numbers"], "pos": r["_positions"], "H": r["hamiltonian"],
                   "S": r.get("overlap"), "energy": r.get("energy"), "forces": r.get("forces")}

    return molecules_to_samples(mols(), "def2_svp_qm7", config, device, convention="orca")


def load_ase_entries(entries, config, device="cpu", basis="def2_tzvpd"):
    """Molecules of ASE databases given as ``{"db_file", "start_idx", "end_idx"}`` segments
    (one rank's share from :func:`maloq_b200.data.asedb.distribute_data`, or a whole file);
    Fock matrices in ``data['fock_matrix']`` are already in e3nn order."""
    from .asedb import ASEDataset

    open_shell = bool(config.get("open_shell", False))

    def mols():
        for e in entries:
            ds = ASEDataset(e["db_file"], open_shell=open_shell, start_idx=e["start_idx"], end_idx=e["end_idx"])
            for i in range(len(ds)):
                r = ds[i]
                yield {"z": r["atomic_numbers"], "pos": r["pos"], "H": r["fock_matrix"], "energy": r["energies"],
                       "charge": r["charge"], "spin": r["spin_multiplicity"]}

    return molecules_to_samples(mols(), _basis_for(basis), config, device, open_shell=open_shell)


def load_omol_csh(path, config, device="cpu", indices=None, opener=None):
    """OMol-CSH-58k HDF5 molecules (def2-TZVPD, order-corrected Fock matrices)."""
    from .omol import OMolCSH58kDatabase

    db = OMolCSH58kDatabase(path, indices=indices, opener=opener)

    def mols():
        for i in range(len(db)):
            r = db[i]
            yield {"z": r["z"], "pos": r["pos"], "H": r["fock"], "charge": r["charge"], "spin": r["spin"] or 1}

    return molecules_to_samples(mols(), _basis_for("def2_tzvpd"), config, device,
                                open_shell=bool(config.get("open_shell", False)))


def _basis_for(name):
    if name == "def2_tzvpd":
        from .omol import def2_tzvpd_by_z

        return def2_tzvpd_by_z()
    return name


def molecules_to_samples(mols, basis, config, device="cpu", convention=None, open_shell=False):
    """Graph samples with coupled-basis Fock targets from molecule dicts with ``z``, ``pos``
    (Angstrom), ``H`` ([n, n], or [2, n, n] alpha/beta) and optionally ``S``, ``energy``,
    ``forces``, ``charge``, ``spin``.  ``convention`` names the code whose orbital order ``H``
    is in (None: already e3nn order).  Closed-shell training keeps the first spin of an
    open-shell matrix; open-shell training repeats a closed-shell matrix for both spins."""
    import torch

    from .basis_sets import get_basis
    from .batch import make_sample
    from .labels import BlockSparseMatrix, orbital_offsets
    from .structures import Structure
    from .targets import FockLabeler

    basis = get_basis(basis)
    labeler = FockLabeler(basis, device=device)
    cutoff = 2 * config.get("rcut_orbitals", 3.0)
    samples = []
    for m in mols:
        Z = np.asarray(m["z"], dtype=np.int64)
        s = make_sample(Structure(Z, np.asarray(m["pos"], dtype=np.float64)), cutoff)
        H = np.asarray(m["H"], dtype=np.float64)
        Hs = H[None] if H.ndim == 2 else H
        if open_shell and Hs.shape[0] == 1:
            Hs = np.concatenate([Hs, Hs])
        elif not open_shell:
            Hs = Hs[:1]
        rows, cols = labeler.pairs(s)
        offs = orbital_offsets(Z, labeler.table)
        nys, ys = [], []
        for Hk in Hs:
            if convention is not None:
                Hk = reorder_orbitals(Hk, Z, basis, convention)
            bsm = BlockSparseMatrix.from_dense(Hk, rows, cols, offs)
            ny, y = labeler.labels_from_blocks(s, bsm)
            nys.append(ny)
            ys.append(y)
        s.node_y, s.y = torch.stack(nys).cpu(), torch.stack(ys).cpu()
        s.overlap = m.get("S")
        if m.get("energy") is not None:
            s.energy = float(np.asarray(m["energy"]).reshape(-1)[0])
        if m.get("forces") is not None:
            s.forces = np.asarray(m["forces"], dtype=np.float64)
        s.charge = int(m.get("charge", 0))
        s.spin = int(m.get("spin", 1)) or 1
        samples.append(s)
    return samples, labeler


# ------------------------------------------------------------------ CP2K (periodic materials)
HARTREE_EV = 27.211386245988
_SYMBOLS = ("X H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge As Se Br "
            "Kr Rb Sr Y Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm Eu Gd Tb Dy Ho Er Tm "
            "Yb Lu Hf Ta W Re Os Ir Pt Au Hg Tl Pb Bi Po At Rn").split()
SYMBOL_TO_Z = {s: i for i, s in enumerate(_SYMBOLS) if i}

# a Fortran unformatted record of (row int32, col int32, value float64): 4-byte length markers
# of 16 around the 16-byte payload
_CP2K_RECORD = np.dtype([("m0", "<i4"), ("row", "<u4"), ("col", "<u4"), ("val", "<f8"), ("m1", "<i4")])


def read_cp2k_csr(path, dtype=np.float64):
    """A CP2K sparse matrix dump (binary Fortran records or ASCII ``row col value`` lines,
    1-based, usually the upper triangle) as a full symmetric ``scipy.sparse`` CSR matrix:
    ``H + H^T - diag(H)``.  Reference ``dataset_utils/get_loader.py:556-622``."""
    import scipy.sparse as sp

    size = os.path.getsize(path)
    rec = None
    if size and size % _CP2K_RECORD.itemsize == 0:
        head = np.fromfile(path, dtype=_CP2K_RECORD, count=min(16, size // _CP2K_RECORD.itemsize))
        if np.all(head["m0"] == 16) and np.all(head["m1"] == 16):
            rec = np.fromfile(path, dtype=_CP2K_RECORD)
    if rec is not None:
        r, c, v = rec["row"].astype(np.int64), rec["col"].astype(np.int64), rec["val"]
    else:
        a = np.loadtxt(path, ndmin=2)
        r, c, v = a[:, 0].astype(np.int64), a[:, 1].astype(np.int64), a[:, 2]
    n = int(max(r.max(), c.max())) if len(r) else 0
    H = sp.coo_matrix((v.astype(dtype), (r - 1, c - 1)), shape=(n, n)).tocsr()
    return (H + H.T - sp.diags(H.diagonal(), format="csr")).tocsr()


def write_cp2k_csr(path, M, binary=True):
    """Write the upper triangle of a (dense or sparse) matrix in CP2K's dump format (tests and
    data export)."""
    import scipy.sparse as sp

    U = sp.triu(sp.coo_matrix(M)).tocoo()
    if binary:
        rec = np.zeros(U.nnz, dtype=_CP2K_RECORD)
        rec["m0"] = rec["m1"] = 16
        rec["row"], rec["col"], rec["val"] = U.row + 1, U.col + 1, U.data
        rec.tofile(path)
    else:
        np.savetxt(path, np.stack([U.row + 1, U.col + 1, U.data], 1), fmt=["%d", "%d", "%.17g"])


def read_periodic_xyz(path):
    """Structure of an XYZ file whose comment line gives the orthorhombic cell as
    ``Lattice="ax ay az bx by bz cx cy cz"`` (diagonal used) / ``Lattice="a b c"`` or as
    ``Cell: a b c`` (CP2K).  Reference ``get_loader.py:644-708``."""
    import re

    from .structures import Structure

    with open(path) as f:
        lines = f.read().splitlines()
    n = int(lines[0].split()[0])
    z, pos = [], []
    for ln in lines[2:2 + n]:
        p = ln.split()
        z.append(SYMBOL_TO_Z[p[0]])
        pos.append([float(x) for x in p[1:4]])
    cell = None
    m = re.search(r'Lattice="([^"]+)"', lines[1])
    if m:
        vals = [float(x) for x in m.group(1).split()]
        cell = [vals[0], vals[4], vals[8]] if len(vals) == 9 else (vals if len(vals) == 3 else None)
    else:
        p = lines[1].split()
        if p and p[0].lower() in ("cell", "cell:"):
            cell = [float(x) for x in p[1:4]]
    return Structure(np.asarray(z, np.int64), np.asarray(pos, np.float64),
                     None if cell is None else np.asarray(cell, np.float64))


def fermi_energy(out_path):
    """Fermi level (Hartree) from a CP2K output file (``Fermi Energy [eV] :`` is converted;
    ``Fermi energy:`` / ``Fermi level:`` are taken as Hartree).  Reference
    ``get_loader.py:710-726``."""
    import re

    pats = [(re.compile(r"Fermi Energy \[eV\] :\s*([-+]?\d*\.?\d+(?:[eE][-+]?\d+)?)"), 1.0 / HARTREE_EV),
            (re.compile(r"Fermi energy:\s*([-+]?\d*\.?\d+(?:[eE][-+]?\d+)?)"), 1.0),
            (re.compile(r"Fermi level:\s*([-+]?\d*\.?\d+(?:[eE][-+]?\d+)?)"), 1.0)]
    with open(out_path) as f:
        for line in f:
            for pat, scale in pats:
                m = pat.search(line)
                if m:
                    return float(m.group(1)) * scale
    raise ValueError(f"no Fermi energy in {out_path}")


def fermi_shift(H, S, mu):
    """H - mu S (the Hamiltonian referenced to the Fermi level)."""
    return H - mu * S


def blocks_from_sparse(M, rows, cols, orb_ptr):
    """:class:`BlockSparseMatrix` of the atom-pair blocks (rows[b], cols[b]) of a sparse
    matrix, without densifying it: each stored entry is mapped to its atom pair and its
    position inside that pair's block (entries of pairs not listed are dropped)."""
    import scipy.sparse as sp

    from .labels import BlockSparseMatrix

    C = sp.coo_matrix(M)
    orb_ptr = np.asarray(orb_ptr, np.int64)
    n_at = len(orb_ptr) - 1
    atom_of = np.repeat(np.arange(n_at), np.diff(orb_ptr))
    rows, cols = np.asarray(rows, np.int64), np.asarray(cols, np.int64)
    norb = np.diff(orb_ptr)
    sizes = norb[rows] * norb[cols]
    ptr = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    data = np.zeros(int(ptr[-1]), dtype=C.dtype)
    key = rows * n_at + cols
    order = np.argsort(key)
    ai, aj = atom_of[C.row], atom_of[C.col]
    k = ai * n_at + aj
    at = np.searchsorted(key[order], k)
    at = np.minimum(at, len(order) - 1)
    hit = key[order][at] == k
    b = order[at[hit]]
    r, c = C.row[hit] - orb_ptr[ai[hit]], C.col[hit] - orb_ptr[aj[hit]]
    data[ptr[b] + r * norb[cols[b]] + c] = C.data[hit]
    return BlockSparseMatrix(rows, cols, ptr, data, orb_ptr)


def load_cp2k(xyz_path, h_path, config, basis_name="dzvp_like", s_path=None, out_path=None, device="cpu"):
    """One periodic CP2K structure with coupled-basis targets: structure from the XYZ, the
    Hamiltonian from the CSR dump (Fermi-shifted, H - mu S, when the overlap and the output
    file are given), graph within 2 * rcut_orbitals, blocks of every graph pair.

    ``config['tiling_dims']`` = (n_a, n_b, n_c) replicates the cell into a supercell (weak
    scaling; reference ``fock_targets_batched.py:71-77``): every pair (i, j) of the supercell
    takes the block of the unit-cell pair (i mod n, j mod n), so each copy carries the unit
    cell's targets."""
    from .basis_sets import get_basis
    from .batch import make_sample
    from .labels import BlockSparseMatrix, orbital_offsets
    from .structures import tile_structure
    from .targets import FockLabeler

    st = read_periodic_xyz(xyz_path)
    H = read_cp2k_csr(h_path)
    if s_path is not None and out_path is not None:
        H = fermi_shift(H, read_cp2k_csr(s_path), fermi_energy(out_path))
    labeler = FockLabeler(get_basis(basis_name), device=device)
    tiling = config.get("tiling_dims")
    n0, z0 = len(st.z), st.z
    if tiling is not None and any(int(d) != 1 for d in tiling):
        st = tile_structure(st, tiling)
    s = make_sample(st, 2 * config.get("rcut_orbitals", 4.0))
    rows, cols = labeler.pairs(s)
    if len(st.z) == n0:
        bsm = blocks_from_sparse(H, rows, cols, orbital_offsets(st.z, labeler.table))
    else:
        key = (np.asarray(rows) % n0) * n0 + np.asarray(cols) % n0
        uk, inv = np.unique(key, return_inverse=True)
        ob = blocks_from_sparse(H, uk // n0, uk % n0, orbital_offsets(z0, labeler.table))
        lens = np.diff(ob.block_ptr)[inv]
        ptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        src = np.arange(int(ptr[-1])) - np.repeat(ptr[:-1], lens) + np.repeat(ob.block_ptr[inv], lens)
        bsm = BlockSparseMatrix(np.asarray(rows, np.int64), np.asarray(cols, np.int64), ptr, ob.data[src],
                                orbital_offsets(st.z, labeler.table))
    ny, y = labeler.labels_from_blocks(s, bsm)
    s.node_y, s.y = ny.unsqueeze(0).cpu(), y.unsqueeze(0).cpu()
    return s, labeler


# ------------------------------------------------------------------ ORCA output
_L_OF = {"s": 0, "p": 1, "d": 2, "f": 3, "g": 4}


def _read_printed_matrix(lines, start, n):
    """An n x n matrix printed in ORCA's column blocks (a header line of column indices, then
    ``row v v v ...`` lines) from ``lines[start]`` (the first header) to the next blank line;
    returns (matrix, index of the blank line)."""
    M = np.zeros((n, n))
    cols = None
    i = start
    while i < len(lines) and lines[i].split():
        parts = lines[i].split()
        if cols is not None and len(parts) == len(cols) + 1 and "." in parts[-1]:
            M[int(parts[0]), cols] = [float(x) for x in parts[1:]]
        else:
            cols = [int(x) for x in parts]
        i += 1
    return M, i


def read_orca_output(path, unrestricted=False):
    """Structure, contracted basis, Fock matrix and total energy from an ORCA output file.

    Returns ``dict(z, pos, basis, fock, energy)``: ``basis`` maps atomic number -> shell l list
    (in ORCA's contracted order, e.g. ``3s2p1d`` -> [0, 0, 0, 1, 1, 2]); ``fock`` is the
    printed ``FOCK`` matrix in ORCA's orbital order (``reorder_orbitals(..., "orca")`` converts
    it), or ``{"alpha", "beta"}`` when ``unrestricted``; ``energy`` is the total SCF energy in
    Hartree (None if absent).  Reference ``fock_utils/utils_orca_out.py:30-50, 282-400``."""
    import re

    with open(path) as f:
        lines = f.read().splitlines()
    z, pos, basis, focks, energy = [], [], {}, [], None
    group = re.compile(r"Group\s+\d+\s+Type\s+(\w+)\s*:\s*\S+\s+contracted to\s+(\S+)")
    i = 0
    while i < len(lines):
        ln = lines[i]
        if "CARTESIAN COORDINATES (ANGSTROEM)" in ln and not z:
            j = i + 2
            while j < len(lines) and lines[j].split():
                p = lines[j].split()
                z.append(SYMBOL_TO_Z[p[0]])
                pos.append([float(x) for x in p[1:4]])
                j += 1
            i = j
            continue
        m = group.search(ln)
        if m:
            shells = []
            for cnt, l in re.findall(r"(\d+)([spdfg])", m.group(2)):
                shells += [_L_OF[l]] * int(cnt)
            basis[SYMBOL_TO_Z[m.group(1)]] = shells
        if "TOTAL SCF ENERGY" in ln:
            for k in range(i + 1, min(i + 10, len(lines))):
                p = lines[k].split()
                if "Total Energy" in lines[k] and "Eh" in p:
                    energy = float(p[p.index("Eh") - 1])
                    break
        if ln.strip() == "FOCK" and not focks:
            n = sum(sum(2 * l + 1 for l in basis[a]) for a in z)
            j = i + 1
            while not lines[j].split() or set(lines[j].strip()) <= {"-"}:
                j += 1
            M, j = _read_printed_matrix(lines, j, n)
            focks.append(M)
            if unrestricted:
                while j < len(lines) and not lines[j].split():
                    j += 1
                M, j = _read_printed_matrix(lines, j, n)
                focks.append(M)
            i = j
            continue
        i += 1
    fock = None
    if focks:
        fock = {"alpha": focks[0], "beta": focks[1]} if unrestricted else focks[0]
    eps, occ = _orbital_energies(lines)
    return {"z": np.asarray(z, np.int64), "pos": np.asarray(pos), "basis": basis, "fock": fock, "energy": energy,
            "orbital_energies": eps, "occupations": occ}


def _orbital_energies(lines):
    """Orbital energies [Eh] and occupations of the last ``ORBITAL ENERGIES`` section: one
    array per spin channel (two after ``SPIN UP`` / ``SPIN DOWN ORBITALS`` headers)."""
    starts = [i for i, ln in enumerate(lines) if ln.strip() == "ORBITAL ENERGIES"]
    if not starts:
        return [], []
    eps, occ = [], []
    i = starts[-1] + 1
    while i < len(lines) and len(eps) < 2:
        t = lines[i].strip()
        if t.split()[:2] == ["NO", "OCC"]:
            e, o = [], []
            i += 1
            while i < len(lines):
                q = lines[i].split()
                try:
                    o.append(float(q[1]))
                    e.append(float(q[2]))
                except (IndexError, ValueError):
                    break
                i += 1
            eps.append(np.asarray(e))
            occ.append(np.asarray(o))
            continue
        # between the tables only blank lines, dashes and the spin headers
        if eps and t and not t.startswith("SPIN") and set(t) != {"-"}:
            break
        i += 1
    return eps, occ


def homo_lumo_energies(orbital_energies, n_electrons, multiplicity=1):
    """(HOMO energies, LUMO energies), one per spin channel: n_alpha = (N + M - 1) / 2 and
    n_beta = (N - M + 1) / 2 occupied orbitals for multiplicity M (reference
    ``utils_orca_out.py:258-269``); a single channel gives the closed-shell / alpha values."""
    n_alpha = (n_electrons + multiplicity - 1) // 2
    homo, lumo = [orbital_energies[0][n_alpha - 1]], [orbital_energies[0][n_alpha]]
    if len(orbital_energies) > 1:
        n_beta = (n_electrons - multiplicity + 1) // 2
        homo.append(orbital_energies[1][n_beta - 1])
        lumo.append(orbital_energies[1][n_beta])
    return homo, lumo


def charge_and_multiplicity_from_path(path, levels=3):
    """(charge, multiplicity) from a run folder named ``..._<charge>_<multiplicity>``, looking at
    the file's folder and up to ``levels - 1`` parents; (0, 1) when none matches (reference
    ``utils_orca_out.py:82-117``)."""
    import re

    d = os.path.dirname(os.path.abspath(path))
    for _ in range(levels):
        m = re.search(r"_(-?\d+)_(\d+)$", os.path.basename(d))
        if m:
            return int(m.group(1)), int(m.group(2))
        parent = os.path.dirname(d)
        if parent == d:
            break
        d = parent
    return 0, 1


def read_finalms(path):
    """The ``finalms`` value of an ORCA input file (final spin projection), or None."""
    import re

    with open(path) as f:
        for ln in f:
            m = re.search(r"finalms\s+([-\d.]+)", ln, re.IGNORECASE)
            if m:
                return float(m.group(1))
    return None


def orbital_count(z, basis):
    """Number of orbitals (the Fock matrix size) of atoms ``z`` in ``basis``."""
    return int(sum(sum(2 * (l % 10) + 1 for l in basis[int(a)]) for a in z))


def sort_by_l(H, basis, z):
    """Reorder each atom's shells by angular momentum (stable within a degree), rows and
    columns (reference ``utils_orca_out.py:467-495``)."""
    perm, off = [], 0
    for a in z:
        shells = []
        for l in basis[int(a)]:
            n = 2 * (l % 10) + 1
            shells.append((l % 10, off, n))
            off += n
        for _, o, n in sorted(shells, key=lambda t: t[0]):
            perm.extend(range(o, o + n))
    return H[np.ix_(perm, perm)]
