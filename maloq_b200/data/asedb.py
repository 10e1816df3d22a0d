"""ASE-database datasets read with the standard-library ``sqlite3`` (no ``ase`` import).

An ASE ``.db`` file is an SQLite database whose ``systems`` table holds one structure per
row: ``numbers`` (int32 blob), ``positions`` (float64 blob, N x 3), ``cell`` (float64 3 x 3),
``pbc`` (bit mask), calculated ``energy`` / ``forces``, ``key_value_pairs`` (JSON text) and
``data`` (a Python object: JSON text in old files, the binary object layout in newer ones -
an int64 offset, then the raw bytes of every array, then JSON in which each array is
``{"__ndarray__": [shape, dtype, byte offset]}``).  This module reads and writes that layout
(it is ASE's file format, kept as is so that files made by ASE load here and files written
here load in ASE).

* :class:`AseDb` - row access: ``count()``, ``rows(start, end)``.
* :class:`ASEDataset` - rows -> molecule dicts with the reference's fields
  (``pos``, ``atomic_numbers``, ``fock_matrix``, ``energies``, ``charge``,
  ``spin_multiplicity``, ``folder_name``), open/closed-shell handling as in the reference
  (``dataset_utils/ASEDataset.py:21-121``).
* :class:`ASEAtomsData` - schnetpack-style rows (``_atomic_numbers``, ``_positions``, ``_cell``,
  ``_pbc``, ``_n_atoms`` plus every ``data`` property), the form the QM7 Hamiltonian database
  takes (reference ``ASEDataset.py:469-832``).
* :func:`get_rank_range` / :func:`distribute_data` - a balanced split of the first
  ``N_train`` (then ``N_val``) molecules of a folder of ``.db`` files over the ranks, mapped
  back to (file, local start, local end) segments (reference ``ASEDataset.py:134-300``).
* :func:`write_asedb` - writes rows in the same layout (tests, database builders).
"""

from __future__ import annotations

import json
import os
import sqlite3
import time

import numpy as np

_SYSTEMS_COLUMNS = (
    "id INTEGER PRIMARY KEY AUTOINCREMENT, unique_id TEXT UNIQUE, ctime REAL, mtime REAL, username TEXT, "
    "numbers BLOB, positions BLOB, cell BLOB, pbc INTEGER, initial_magmoms BLOB, initial_charges BLOB, "
    "masses BLOB, tags BLOB, momenta BLOB, constraints TEXT, calculator TEXT, calculator_parameters TEXT, "
    "energy REAL, free_energy REAL, forces BLOB, stress BLOB, dipole BLOB, magmoms BLOB, magmom REAL, "
    "charges BLOB, key_value_pairs TEXT, data BLOB, natoms INTEGER, fmax REAL, smax REAL, volume REAL, "
    "mass REAL, charge REAL")
_FORMAT_VERSION = 9  # the newest layout this module writes (binary ``data``)


# ------------------------------------------------------------------ object (de)serialisation
def _from_binary(buf):
    """Decode the binary object layout (int64 JSON offset, array bytes, JSON)."""
    buf = bytes(buf)
    off = int(np.frombuffer(buf[:8], "<i8")[0])
    return _restore(json.loads(buf[off:].decode()), buf)


def _restore(obj, buf):
    if isinstance(obj, list):
        return [_restore(v, buf) for v in obj]
    if not isinstance(obj, dict):
        return obj
    if "__complex__" in obj:
        re, im = obj["__complex__"]
        return complex(re, im)
    if "__ndarray__" in obj:
        shape, dtype, where = obj["__ndarray__"]
        dt = np.dtype(dtype)
        if isinstance(where, list):  # JSON text layout: the values themselves
            if dt.kind == "c":
                a = np.asarray(where, dtype=float).view(dt)
            else:
                a = np.asarray(where, dtype=dt)
            return a.reshape(shape)
        n = int(np.prod(shape)) if len(shape) else 1
        a = np.frombuffer(buf[where:where + n * dt.itemsize], dt.newbyteorder("<")).copy()
        return a.reshape(shape)
    return {k: _restore(v, buf) for k, v in obj.items()}


def _to_binary(obj):
    """Encode ``obj`` (dicts, lists, numbers, strings, numpy arrays) in the binary layout."""
    parts = [b"\0" * 8]

    def enc(o):
        if isinstance(o, dict):
            return {str(k): enc(v) for k, v in o.items()}
        if isinstance(o, (list, tuple)):
            return [enc(v) for v in o]
        if isinstance(o, np.ndarray):
            o = np.ascontiguousarray(o)
            if o.dtype == object:
                raise TypeError("object arrays cannot be stored")
            off = sum(len(p) for p in parts)
            parts.append(o.astype(o.dtype.newbyteorder("<"), copy=False).tobytes())
            return {"__ndarray__": [list(o.shape), o.dtype.name, off]}
        if isinstance(o, np.generic):
            return o.item()
        if isinstance(o, complex):
            return {"__complex__": [o.real, o.imag]}
        return o

    tree = enc(obj)
    off = sum(len(p) for p in parts)
    parts[0] = np.asarray(off, "<i8").tobytes()
    parts.append(json.dumps(tree, separators=(",", ":")).encode())
    return b"".join(parts)


def _decode_data(v):
    if v is None:
        return {}
    if isinstance(v, (bytes, memoryview)):
        b = bytes(v)
        if b[:1] in (b"{", b"["):  # JSON stored as a blob
            return _restore(json.loads(b.decode()), b)
        return _from_binary(b)
    return _restore(json.loads(v), b"")


def _blob(buf, dtype, shape=None):
    if buf is None:
        return None
    a = np.frombuffer(bytes(buf), np.dtype(dtype).newbyteorder("<")).copy()
    return a.reshape(shape) if shape is not None else a


# ------------------------------------------------------------------ database access
class AseDb:
    """Read-only rows of an ASE SQLite database (``systems`` table)."""

    def __init__(self, path):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        self.conn = sqlite3.connect(f"file:{path}?mode=ro", uri=True)
        cols = [r[1] for r in self.conn.execute("PRAGMA table_info(systems)")]
        if not cols:
            raise ValueError(f"{path} is not an ASE database (no systems table)")
        self._cols = cols

    def count(self):
        return int(self.conn.execute("SELECT COUNT(*) FROM systems").fetchone()[0])

    def _row(self, values):
        r = dict(zip(self._cols, values))
        n = r.get("natoms")
        numbers = _blob(r["numbers"], np.int32)
        natoms = len(numbers) if numbers is not None else int(n or 0)
        pbc = int(r.get("pbc") or 0)
        return {
            "id": r["id"],
            "numbers": numbers.astype(np.int64) if numbers is not None else np.zeros(0, np.int64),
            "positions": _blob(r["positions"], np.float64, (natoms, 3)),
            "cell": _blob(r.get("cell"), np.float64, (3, 3)),
            "pbc": np.array([(pbc >> i) & 1 for i in range(3)], dtype=bool),
            "energy": r.get("energy"),
            "forces": _blob(r.get("forces"), np.float64, (natoms, 3)),
            "charge": r.get("charge"),
            "key_value_pairs": json.loads(r["key_value_pairs"]) if r.get("key_value_pairs") else {},
            "data": _decode_data(r.get("data")),
        }

    def rows(self, start=0, end=None):
        """Rows ``start .. end-1`` in id order, as dicts."""
        end = self.count() if end is None else end
        cur = self.conn.execute("SELECT * FROM systems ORDER BY id LIMIT ? OFFSET ?", (max(0, end - start), start))
        return [self._row(v) for v in cur]

    def close(self):
        self.conn.close()


def write_asedb(path, rows, binary=True):
    """Write ``rows`` (dicts with ``numbers``, ``positions`` and optionally ``cell``, ``pbc``,
    ``energy``, ``forces``, ``charge``, ``key_value_pairs``, ``data``) as an ASE database.
    ``binary=False`` stores ``data`` as JSON text (the older layout)."""
    conn = sqlite3.connect(path)
    conn.execute(f"CREATE TABLE IF NOT EXISTS systems ({_SYSTEMS_COLUMNS})")
    conn.execute("CREATE TABLE IF NOT EXISTS information (name TEXT, value TEXT)")
    if conn.execute("SELECT COUNT(*) FROM information").fetchone()[0] == 0:
        conn.execute("INSERT INTO information VALUES ('version', ?)", (str(_FORMAT_VERSION if binary else 8),))
    now = time.time()
    for r in rows:
        numbers = np.asarray(r["numbers"], np.int32)
        pos = np.asarray(r["positions"], np.float64).reshape(-1, 3)
        cell = np.asarray(r.get("cell", np.zeros((3, 3))), np.float64).reshape(3, 3)
        pbc = r.get("pbc", (False, False, False))
        pbc_bits = int(sum(int(bool(p)) << i for i, p in enumerate(pbc)))
        forces = r.get("forces")
        data = r.get("data") or {}
        if binary:
            data_col = sqlite3.Binary(_to_binary(data))
        else:
            def js(o):
                if isinstance(o, np.ndarray):
                    return {"__ndarray__": [list(o.shape), o.dtype.name, o.ravel().tolist()]}
                if isinstance(o, dict):
                    return {k: js(v) for k, v in o.items()}
                if isinstance(o, (list, tuple)):
                    return [js(v) for v in o]
                return o.item() if isinstance(o, np.generic) else o
            data_col = json.dumps(js(data))
        conn.execute(
            "INSERT INTO systems (unique_id, ctime, mtime, username, numbers, positions, cell, pbc, energy, forces, "
            "key_value_pairs, data, natoms, charge) VALUES (?,?,?,?,?,?,?,?,?,?,?,?,?,?)",
            (os.urandom(16).hex(), now, now, "maloq", numbers.tobytes(), pos.tobytes(), cell.tobytes(), pbc_bits,
             None if r.get("energy") is None else float(r["energy"]),
             None if forces is None else np.asarray(forces, np.float64).tobytes(),
             json.dumps(r.get("key_value_pairs", {})), data_col, len(numbers),
             None if r.get("charge") is None else float(r["charge"])))
    conn.commit()
    conn.close()


# ------------------------------------------------------------------ datasets
class ASEDataset:
    """Molecules of one ASE database with Fock-matrix targets in ``data['fock_matrix']``
    (and ``'total_energy [Eh]'``, ``'is_open_shell'``, ``'charge'``, ``'spin_multiplicity'``,
    ``'folder_name'``).  Rows ``start_idx .. end_idx-1`` are kept.  In open-shell training a
    closed-shell matrix is repeated for both spins; in closed-shell training an open-shell
    molecule keeps its alpha matrix."""

    def __init__(self, db_path, dtype=np.float32, open_shell=False, start_idx=0, end_idx=None):
        self.db_path, self.open_shell = db_path, open_shell
        self.dtype = np.float32 if str(dtype).endswith("float32") else np.float64
        db = AseDb(db_path)
        try:
            self.rows = db.rows(start_idx, end_idx)
        finally:
            db.close()

    def __len__(self):
        return len(self.rows)

    def __getitem__(self, idx):
        r = self.rows[idx]
        d = r["data"]
        fock = np.asarray(d["fock_matrix"], dtype=self.dtype)
        is_os = bool(d.get("is_open_shell", False))
        charge, spin = (int(d.get("charge", 0)), int(d.get("spin_multiplicity", 1))) if is_os else (0, 1)
        if self.open_shell and not is_os:
            fock = np.repeat(fock[None], 2, axis=0)
        elif not self.open_shell and is_os:
            fock = fock[0]
        return {"pos": r["positions"], "atomic_numbers": r["numbers"], "fock_matrix": fock,
                "energies": d.get("total_energy [Eh]", r["energy"]), "num_atoms_in_molecule": len(r["numbers"]),
                "charge": charge, "spin_multiplicity": spin, "folder_name": d.get("folder_name", "")}


class ASEAtomsData:
    """Schnetpack-style rows of an ASE database: structure fields under ``_atomic_numbers``,
    ``_positions``, ``_cell``, ``_pbc``, ``_n_atoms``, and every array of the row's ``data``
    under its own name (e.g. ``hamiltonian``, ``overlap``, ``energy``, ``forces`` in the
    QM7 Hamiltonian database).  Property arrays stored flat are reshaped: square matrices
    to (n, n), per-atom vectors to (N, 3)."""

    def __init__(self, datapath, load_properties=None):
        self.datapath = datapath
        self.load_properties = load_properties
        db = AseDb(datapath)
        try:
            self._n = db.count()
        finally:
            db.close()
        self._db = None

    def __len__(self):
        return self._n

    def _conn(self):
        if self._db is None:
            self._db = AseDb(self.datapath)
        return self._db

    def __getitem__(self, idx):
        if idx < 0 or idx >= self._n:
            raise IndexError(idx)
        r = self._conn().rows(idx, idx + 1)[0]
        n = len(r["numbers"])
        out = {"_idx": idx, "_n_atoms": n, "_atomic_numbers": r["numbers"], "_positions": r["positions"],
               "_cell": r["cell"], "_pbc": r["pbc"]}
        for k, v in r["data"].items():
            if self.load_properties is not None and k not in self.load_properties:
                continue
            v = np.asarray(v)
            while v.ndim >= 2 and v.shape[0] == 1:  # per-row batch axis
                v = v[0]
            if v.ndim == 1 and k == "forces" and v.size == 3 * n:
                v = v.reshape(n, 3)
            elif v.ndim == 1 and v.size > 1 and int(round(v.size ** 0.5)) ** 2 == v.size and k != "forces":
                m = int(round(v.size ** 0.5))
                v = v.reshape(m, m)
            out[k] = v
        if "energy" not in out and r["energy"] is not None:
            out["energy"] = np.array([r["energy"]])
        if "forces" not in out and r["forces"] is not None:
            out["forces"] = r["forces"]
        return out


def get_rank_range(total_count, world_size, rank, global_offset=0):
    """[start, end) of ``rank``'s share of ``total_count`` items: the first
    ``total_count % world_size`` ranks get one extra item."""
    avg, rem = divmod(total_count, world_size)
    size = avg + 1 if rank < rem else avg
    start = rank * (avg + 1) if rank < rem else rem * (avg + 1) + (rank - rem) * avg
    return global_offset + start, global_offset + start + size


def db_files_in(base_folder):
    folders = [base_folder] if isinstance(base_folder, str) else list(base_folder)
    out = []
    for f in folders:
        out += sorted(os.path.join(f, x) for x in os.listdir(f) if x.endswith(".db"))
    return out


def distribute_data(base_folder, world_size, rank, N_global_train, N_global_val):
    """This rank's training and validation segments of a folder (or folders) of ``.db`` files.

    The files are concatenated (sorted by name) into one global index space; the first
    ``N_global_train`` molecules are the training set and the next ``N_global_val`` the
    validation set; each set is split over the ranks by :func:`get_rank_range`; the rank's
    global ranges are cut at file boundaries.  Returns (train_entries, val_entries), lists of
    ``{"db_file", "start_idx", "end_idx"}`` with file-local indices."""
    files = []
    g = 0
    for path in db_files_in(base_folder):
        try:
            db = AseDb(path)
            n = db.count()
            db.close()
        except (sqlite3.Error, ValueError):
            n = 0
        if n > 0:
            files.append((path, g, g + n))
            g += n
    if N_global_train + N_global_val > g:
        raise ValueError(f"requested {N_global_train + N_global_val} molecules, the databases hold {g}")

    def segments(lo, hi, limit_lo, limit_hi):
        out = []
        for path, f0, f1 in files:
            a, b = max(lo, f0, limit_lo), min(hi, f1, limit_hi)
            if a < b:
                out.append({"db_file": path, "start_idx": a - f0, "end_idx": b - f0})
        return out

    t0, t1 = get_rank_range(N_global_train, world_size, rank, 0)
    v0, v1 = get_rank_range(N_global_val, world_size, rank, N_global_train)
    return (segments(t0, t1, 0, N_global_train),
            segments(v0, v1, N_global_train, N_global_train + N_global_val))
