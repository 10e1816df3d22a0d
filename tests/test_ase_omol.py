"""ASE-database and OMol-CSH data paths on generated files (CPU): the ASE SQLite layout
(binary and JSON ``data``), schnetpack-style QM7 rows, rank ranges over folders of
databases, the OMol diffuse-order fix, and the workflow training on each source."""
import json
import os

import numpy as np
import pytest
import torch

from maloq_b200.data import asedb, omol, readers
from maloq_b200.data.basis_sets import get_basis, n_orbitals


def _mol(rng, basis, elements=(1, 6, 8), n=4, open_shell=False):
    z = rng.choice(elements, size=n)
    pos = rng.uniform(0, 3.0, size=(n, 3))
    norb = sum(n_orbitals(basis, int(a)) for a in z)
    H = rng.normal(size=(norb, norb))
    H = H + H.T
    if open_shell:
        H = np.stack([H, H + 0.1 * np.eye(norb)])
    return z, pos, H


@pytest.mark.parametrize("binary", [True, False])
def test_asedb_roundtrip(tmp_path, binary):
    rng = np.random.default_rng(0)
    rows = []
    for i in range(5):
        z, pos, H = _mol(rng, get_basis("def2_svp_qm7"))
        rows.append({"numbers": z, "positions": pos, "energy": -1.5 * i, "forces": rng.normal(size=(len(z), 3)),
                     "pbc": (True, False, True), "cell": np.diag([5.0, 6.0, 7.0]),
                     "key_value_pairs": {"tag": i},
                     "data": {"fock_matrix": H.astype(np.float32), "total_energy [Eh]": -2.0 * i,
                              "is_open_shell": False, "folder_name": f"m{i}", "nested": {"v": np.arange(3)}}})
    path = str(tmp_path / "x.db")
    asedb.write_asedb(path, rows, binary=binary)
    db = asedb.AseDb(path)
    assert db.count() == 5
    got = db.rows(1, 4)
    assert [g["key_value_pairs"]["tag"] for g in got] == [1, 2, 3]
    g = got[1]
    assert np.array_equal(g["numbers"], rows[2]["numbers"]) and np.allclose(g["positions"], rows[2]["positions"])
    assert g["pbc"].tolist() == [True, False, True] and np.allclose(g["cell"], np.diag([5.0, 6.0, 7.0]))
    assert np.allclose(g["forces"], rows[2]["forces"]) and g["energy"] == -3.0
    assert np.array_equal(g["data"]["fock_matrix"], rows[2]["data"]["fock_matrix"])
    assert g["data"]["fock_matrix"].dtype == np.float32
    assert np.array_equal(g["data"]["nested"]["v"], np.arange(3))
    ds = asedb.ASEDataset(path, start_idx=2, end_idx=5)
    assert len(ds) == 3 and ds[0]["folder_name"] == "m2" and ds[0]["energies"] == -4.0
    os_ds = asedb.ASEDataset(path, open_shell=True, start_idx=0, end_idx=1)
    assert os_ds[0]["fock_matrix"].shape[0] == 2


def test_binary_layout_offsets():
    """The binary ``data`` layout: int64 offset of the JSON, array bytes addressed by offset."""
    b = asedb._to_binary({"a": np.arange(4, dtype=np.int32), "b": [1.5, "s"]})
    off = int(np.frombuffer(b[:8], "<i8")[0])
    tree = json.loads(b[off:].decode())
    shape, dtype, where = tree["a"]["__ndarray__"]
    assert shape == [4] and dtype == "int32" and where == 8
    assert np.array_equal(np.frombuffer(b[where:where + 16], "<i4"), np.arange(4))
    assert asedb._from_binary(b)["b"] == [1.5, "s"]


def test_rank_ranges_cover_every_molecule_once(tmp_path):
    rng = np.random.default_rng(1)
    sizes = [7, 3, 11]
    for k, n in enumerate(sizes):
        rows = [{"numbers": [1, 1], "positions": rng.normal(size=(2, 3)), "data": {"i": k * 100 + i}}
                for i in range(n)]
        asedb.write_asedb(str(tmp_path / f"part{k}.db"), rows)
    (tmp_path / "notes.txt").write_text("not a database")
    for world in (1, 2, 3, 4):
        seen_tr, seen_va = [], []
        for r in range(world):
            lo, hi = asedb.get_rank_range(13, world, r)
            assert hi - lo in (13 // world, 13 // world + 1)
            tr, va = asedb.distribute_data(str(tmp_path), world, r, 13, 6)
            for e, seen in [(x, seen_tr) for x in tr] + [(x, seen_va) for x in va]:
                db = asedb.AseDb(e["db_file"])
                seen += [row["data"]["i"] for row in db.rows(e["start_idx"], e["end_idx"])]
        allrows = [k * 100 + i for k, n in enumerate(sizes) for i in range(n)]
        assert seen_tr == allrows[:13] and seen_va == allrows[13:19]
    with pytest.raises(ValueError):
        asedb.distribute_data(str(tmp_path), 2, 0, 20, 5)


def test_qm7_rows_and_orca_order(tmp_path):
    """Schnetpack-style rows (flat hamiltonian) load as square matrices and are converted from
    ORCA's order; labels -> blocks reproduce the converted matrix."""
    basis = get_basis("def2_svp_qm7")
    rng = np.random.default_rng(2)
    rows, Hs = [], []
    for _ in range(3):
        z, pos, H = _mol(rng, basis, n=3)
        Hs.append((z, H))
        rows.append({"numbers": z, "positions": pos,
                     "data": {"hamiltonian": H.ravel()[None].astype(np.float64), "overlap": np.eye(len(H)),
                              "energy": np.array([-1.0]), "forces": np.zeros(3 * len(z))}})
    path = str(tmp_path / "qm7.db")
    asedb.write_asedb(path, rows)
    d = asedb.ASEAtomsData(path)
    r = d[1]
    assert r["hamiltonian"].shape == Hs[1][1].shape and r["forces"].shape == (3, 3)
    samples, lab = readers.load_qm7(path, {"rcut_orbitals": 10.0})
    s = samples[0]
    dense = lab.blocks_from_labels(s, s.node_y[0], s.y[0]).to_dense()
    assert np.allclose(dense, readers.reorder_orbitals(Hs[0][1], Hs[0][0], basis, "orca"), atol=1e-4)


def test_orca_diffuse_order_fix():
    """A matrix converted with l-sorted shells is restored to the true def2-TZVPD order."""
    basis = omol.def2_tzvpd_by_z()
    z = [8, 1, 6]
    rng = np.random.default_rng(3)
    n = sum(n_orbitals(basis, a) for a in z)
    H_raw = rng.normal(size=(n, n))
    H_raw = H_raw + H_raw.T  # ORCA order
    truth = readers.reorder_orbitals(H_raw, z, basis, "orca")
    sorted_basis = {a: sorted(basis[a]) for a in set(z)}
    corrupted = readers.reorder_orbitals(H_raw, z, sorted_basis, "orca")
    assert not np.allclose(corrupted, truth)
    assert np.allclose(omol.restore_orca_diffuse_order(corrupted, z), truth)
    flat = corrupted[np.triu_indices(n)]
    assert np.allclose(omol.restore_orca_diffuse_order(flat, z), truth)
    assert np.allclose(readers.reorder_orbitals_inverse(truth, z, basis, "orca"), H_raw)


class _Group(dict):
    def __init__(self, d, attrs):
        super().__init__(d)
        self.attrs = attrs


def test_omol_database_with_fake_hdf5(tmp_path):
    basis = omol.def2_tzvpd_by_z()
    rng = np.random.default_rng(4)
    fake, truths = {}, []
    for k in range(3):
        z = np.array([8, 1, 1])
        n = sum(n_orbitals(basis, int(a)) for a in z)
        H_raw = rng.normal(size=(n, n))
        H_raw = H_raw + H_raw.T
        truths.append(readers.reorder_orbitals(H_raw, z, basis, "orca"))
        corrupted = readers.reorder_orbitals(H_raw, z, {a: sorted(basis[a]) for a in set(z.tolist())}, "orca")
        fake[f"mol{k}"] = _Group({"fock": corrupted[np.triu_indices(n)], "elements": z,
                                  "coords": rng.normal(size=(3, 3))}, {"charge": 0, "spin": 1})
    path = str(tmp_path / "omol.h5")
    omol.save_keys_manifest(path, opener=lambda p: fake)
    assert json.load(open(path + ".keys.json")) == ["mol0", "mol1", "mol2"]
    db = omol.OMolCSH58kDatabase(path, indices=[2, 0], opener=lambda p: fake)
    assert len(db) == 2 and db[0]["name"] == "mol2"
    assert np.allclose(db[0]["fock"], truths[2], atol=1e-5)
    samples, lab = readers.load_omol_csh(path, {"rcut_orbitals": 10.0}, indices=[1], opener=lambda p: fake)
    s = samples[0]
    dense = lab.blocks_from_labels(s, s.node_y[0], s.y[0]).to_dense()
    assert np.allclose(dense, truths[1], atol=1e-4)


@pytest.mark.parametrize("source", ["QM7", "folder"])
def test_workflow_trains_on_ase_sources(tmp_path, source):
    from maloq.train_utils import training_workflow

    rng = np.random.default_rng(5)
    if source == "QM7":
        basis = get_basis("def2_svp_qm7")
        rows = []
        for _ in range(6):
            z, pos, H = _mol(rng, basis, n=3)
            rows.append({"numbers": z, "positions": pos, "data": {"hamiltonian": H, "overlap": np.eye(len(H))}})
        path = str(tmp_path / "qm7.db")
        asedb.write_asedb(path, rows)
        extra = dict(dataset_name="QM7", dbpath=path, num_train=4, num_val=2)
    else:
        basis = omol.def2_tzvpd_by_z()
        folder = tmp_path / "dbs"
        folder.mkdir()
        for k in range(2):
            rows = []
            for _ in range(4):
                z, pos, H = _mol(rng, basis, elements=(1, 8), n=3)
                rows.append({"numbers": z, "positions": pos,
                             "data": {"fock_matrix": H, "total_energy [Eh]": -1.0, "is_open_shell": False,
                                      "folder_name": "x"}})
            asedb.write_asedb(str(folder / f"p{k}.db"), rows)
        extra = dict(dataset_name="omol", dbpath=str(folder), num_train=6, num_val=2)
    cfg = dict(batch_size=2, num_epochs=3, l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8,
               rcut_orbitals=3.0, rcut_gaussian=6.0, mmax=2, lr_init=3e-3, output_folder=str(tmp_path / "out"),
               device="cpu", log_every=0, **extra)
    h = training_workflow.TrainingWorkflow(cfg).run()
    assert np.isfinite(h["train_node"][-1]) and h["train_node"][-1] < h["train_node"][0]
    assert os.path.exists(tmp_path / "out" / "backbone.pt")
    torch.manual_seed(0)
