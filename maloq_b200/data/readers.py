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
"""

from __future__ import annotations

import math
import sqlite3

import numpy as np

BOHR_TO_ANGSTROM = 0.52917721092

# code -> shell letter -> (index permutation into e3nn order, signs)
CONVENTIONS = {
    "psi4": {"s": ([0], [1]), "p": ([2, 0, 1], [1, 1, 1]), "d": ([4, 2, 0, 1, 3], [1, 1, 1, 1, 1])},
    "orca": {"s": ([0], [1]), "p": ([2, 0, 1], [1, 1, 1]), "d": ([4, 2, 0, 1, 3], [1, 1, 1, 1, 1])},
    "pyscf": {"s": ([0], [1]), "p": ([1, 2, 0], [1, 1, 1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, 1, 1])},
    "aims": {"s": ([0], [1]), "p": ([0, 1, 2], [1, 1, -1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, -1, 1])},
    "e3nn": {"s": ([0], [1]), "p": ([0, 1, 2], [1, 1, 1]), "d": ([0, 1, 2, 3, 4], [1, 1, 1, 1, 1]),
             "f": ([0, 1, 2, 3, 4, 5, 6], [1] * 7)},
}
_L_LETTER = {0: "s", 1: "p", 2: "d", 3: "f"}


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
    from .basis_sets import get_basis
    from .batch import make_sample
    from .labels import BlockSparseMatrix, orbital_offsets
    from .structures import Structure
    from .targets import FockLabeler

    basis = get_basis("def2_svp_nabla")
    labeler = FockLabeler(basis, device=device)
    db = NablaDFTDatabase(path)
    n = len(db) if indices is None else None
    idx = list(range(min(n, config.get("num_structures", n)))) if indices is None else list(indices)
    cutoff = 2 * config.get("rcut_orbitals", 3.0)
    samples = []
    for i in idx:
        Z, R, E, F, H, S, C = db[i]
        s = make_sample(Structure(Z, R * BOHR_TO_ANGSTROM), cutoff)
        Hs = reorder_orbitals(H.astype(np.float64), Z, basis, convention)
        rows, cols = labeler.pairs(s)
        bsm = BlockSparseMatrix.from_dense(Hs, rows, cols, orbital_offsets(Z, labeler.table))
        ny, y = labeler.labels_from_blocks(s, bsm)
        s.node_y, s.y = ny.unsqueeze(0).cpu(), y.unsqueeze(0).cpu()
        s.overlap = S
        samples.append(s)
    return samples, labeler
