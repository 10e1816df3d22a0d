"""CP2K readers: sparse dumps (binary and ASCII), periodic XYZ headers, Fermi level, block
extraction from sparse matrices, and an end-to-end periodic load."""
import numpy as np
import pytest
import scipy.sparse as sp

from maloq_b200.data import readers, structures
from maloq_b200.data.labels import BlockSparseMatrix, orbital_offsets


@pytest.mark.parametrize("binary", [True, False])
def test_csr_roundtrip_symmetrises(tmp_path, binary):
    rng = np.random.default_rng(0)
    A = sp.random(40, 40, density=0.2, random_state=1).toarray()
    A = A + A.T + np.diag(rng.random(40))
    path = tmp_path / "h.csr"
    readers.write_cp2k_csr(path, A, binary=binary)
    B = readers.read_cp2k_csr(path).toarray()
    assert np.allclose(A, B, atol=1e-12)


def test_periodic_xyz_headers_and_fermi(tmp_path):
    body = "3\n{}\nSi 0 0 0\nO 1.6 0 0\nHf 0 1.9 0.5\n"
    p1 = tmp_path / "a.xyz"
    p1.write_text(body.format('Lattice="10 0 0 0 11 0 0 0 12" Properties=species:S:1:pos:R:3'))
    p2 = tmp_path / "b.xyz"
    p2.write_text(body.format("Cell: 10 11 12"))
    for p in (p1, p2):
        s = readers.read_periodic_xyz(p)
        assert list(s.z) == [14, 8, 72]
        assert np.allclose(s.cell, [10, 11, 12])
    out = tmp_path / "cp2k.out"
    out.write_text("junk\n Fermi Energy [eV] :   -4.747024\n")
    assert abs(readers.fermi_energy(out) - (-4.747024 / readers.HARTREE_EV)) < 1e-12
    H, S = sp.identity(3, format="csr") * 2.0, sp.identity(3, format="csr")
    assert np.allclose(readers.fermi_shift(H, S, 0.5).toarray(), 1.5 * np.eye(3))


def test_blocks_from_sparse_equal_dense_path():
    from maloq_b200.data import datasets
    from maloq_b200.data.batch import make_sample

    rng = np.random.default_rng(1)
    st = structures.amorphous_sio2(rng, 60)
    lab = datasets.labeler_for("sio2")
    s = make_sample(structures.Structure(st.z, st.pos, st.cell * 0 + 17.0), 6.0)
    rows, cols = lab.pairs(s)
    orb = orbital_offsets(s.z, lab.table)
    M = rng.standard_normal((orb[-1], orb[-1]))
    M[np.abs(M) < 1.0] = 0.0
    a = readers.blocks_from_sparse(sp.csr_matrix(M), rows, cols, orb)
    b = BlockSparseMatrix.from_dense(M, rows, cols, orb)
    assert np.array_equal(a.block_ptr, b.block_ptr) and np.allclose(a.data, b.data)


def test_load_cp2k_end_to_end(tmp_path):
    rng = np.random.default_rng(2)
    st = structures.amorphous_sio2(rng, 120)
    cell = np.full(3, 17.0)
    sym = {14: "Si", 8: "O"}
    lines = [str(len(st.z)), "Cell: 17 17 17"] + [f"{sym[int(z)]} {p[0]:.6f} {p[1]:.6f} {p[2]:.6f}"
                                                 for z, p in zip(st.z, np.mod(st.pos, cell))]
    (tmp_path / "s.xyz").write_text("\n".join(lines) + "\n")
    n = 13 * len(st.z)
    A = sp.random(n, n, density=0.01, random_state=3)
    A = (A + A.T).tocsr()
    readers.write_cp2k_csr(tmp_path / "h.csr", A)
    s, lab = readers.load_cp2k(tmp_path / "s.xyz", tmp_path / "h.csr", {"rcut_orbitals": 4.0})
    assert s.node_y.shape == (1, s.num_nodes, lab.target_len)
    assert s.y.shape == (1, s.num_edges, lab.target_len)
    # coupled labels -> blocks -> the dumped matrix entries of those pairs
    back = lab.blocks_from_labels(s, s.node_y[0], s.y[0])
    ref = readers.blocks_from_sparse(A, back.rows, back.cols, back.orb_ptr)
    assert np.allclose(back.data, ref.data, atol=1e-5)


def test_workflow_trains_on_a_cp2k_folder(tmp_path):
    from maloq.train_utils import training_workflow

    rng = np.random.default_rng(4)
    sym = {14: "Si", 8: "O"}
    for k in range(2):
        d = tmp_path / "data" / f"s{k}"
        d.mkdir(parents=True)
        st = structures.amorphous_sio2(rng, 60)
        cell = np.full(3, 13.0)
        lines = [str(len(st.z)), "Cell: 13 13 13"] + [f"{sym[int(z)]} {p[0]:.6f} {p[1]:.6f} {p[2]:.6f}"
                                                     for z, p in zip(st.z, np.mod(st.pos * 13.0 / st.cell, cell))]
        (d / "structure.xyz").write_text("\n".join(lines) + "\n")
        n = 13 * len(st.z)
        A = sp.random(n, n, density=0.02, random_state=k)
        readers.write_cp2k_csr(d / "hamiltonian.csr", (A + A.T).tocsr())
    cfg = dict(dataset_name="cp2k", dbpath=str(tmp_path / "data"), batch_size=1, num_epochs=2, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=3.0, rcut_gaussian=6.0, mmax=2,
               output_folder=str(tmp_path / "out"), device="cpu", log_every=0)
    h = training_workflow.TrainingWorkflow(cfg).run()
    assert len(h["train_node"]) == 2 and np.isfinite(h["train_node"][-1])


def _orca_block(M, width=6):
    out = []
    n = len(M)
    for c0 in range(0, n, width):
        cols = list(range(c0, min(n, c0 + width)))
        out.append("                  " + "    ".join(f"{c:6d}" for c in cols))
        for r in range(n):
            out.append(f"{r:6d}  " + "  ".join(f"{M[r, c]:10.6f}" for c in cols))
    return out


@pytest.mark.parametrize("unrestricted", [False, True])
def test_orca_output_reader(tmp_path, unrestricted):
    rng = np.random.default_rng(5)
    n = 5 + 14  # H (2s1p) + O (3s2p1d)
    Fa = np.round(rng.standard_normal((n, n)), 6)
    Fb = np.round(rng.standard_normal((n, n)), 6)
    lines = ["junk", "---------------------------------", "CARTESIAN COORDINATES (ANGSTROEM)",
             "---------------------------------", "  H      0.000000    0.000000    0.740000",
             "  O      0.100000   -0.200000    0.000000", "", " BASIS SET INFORMATION",
             "Group   1 Type H   : 4s1p contracted to 2s1p pattern {31/1}",
             "Group   2 Type O   : 7s4p1d contracted to 3s2p1d pattern {511/31/1}", "",
             "TOTAL SCF ENERGY", "----------------", "",
             "Total Energy       :        -76.40123456789 Eh           -2078.97 eV", "", "FOCK", ""]
    lines += _orca_block(Fa) + ([""] + _orca_block(Fb) if unrestricted else []) + ["", "end"]
    p = tmp_path / "orca.out"
    p.write_text("\n".join(lines) + "\n")
    d = readers.read_orca_output(p, unrestricted=unrestricted)
    assert list(d["z"]) == [1, 8] and np.allclose(d["pos"][1], [0.1, -0.2, 0.0])
    assert d["basis"] == {1: [0, 0, 1], 8: [0, 0, 0, 1, 1, 2]}
    assert abs(d["energy"] + 76.40123456789) < 1e-12
    if unrestricted:
        assert np.allclose(d["fock"]["alpha"], Fa) and np.allclose(d["fock"]["beta"], Fb)
    else:
        assert np.allclose(d["fock"], Fa)


def test_tiled_cell_matches_the_unit_cell_per_copy(tmp_path):
    """tiling_dims: every copy of the supercell carries the unit cell's node labels, and every
    supercell edge the labels of its unit-cell pair (cutoff below half the cell, so each
    pair has one image)."""
    rng = np.random.default_rng(4)
    st = structures.amorphous_sio2(rng, 90)
    L = 17.0
    sym = {14: "Si", 8: "O"}
    lines = [str(len(st.z)), f"Cell: {L} {L} {L}"] + [f"{sym[int(z)]} {p[0]:.6f} {p[1]:.6f} {p[2]:.6f}"
                                                     for z, p in zip(st.z, np.mod(st.pos, L))]
    (tmp_path / "s.xyz").write_text("\n".join(lines) + "\n")
    n_orb = 13 * len(st.z)
    A = sp.random(n_orb, n_orb, density=0.02, random_state=5)
    A = (A + A.T).tocsr()
    readers.write_cp2k_csr(tmp_path / "h.csr", A)
    cfg = {"rcut_orbitals": 3.0}
    s1, lab = readers.load_cp2k(tmp_path / "s.xyz", tmp_path / "h.csr", cfg)
    s2, _ = readers.load_cp2k(tmp_path / "s.xyz", tmp_path / "h.csr", dict(cfg, tiling_dims=[2, 1, 3]))
    n = s1.num_nodes
    assert s2.num_nodes == 6 * n and s2.num_edges == 6 * s1.num_edges
    for c in range(6):
        assert np.allclose(s2.node_y[0][c * n:(c + 1) * n].numpy(), s1.node_y[0].numpy())
    ref = {(int(i), int(j)): k for k, (i, j) in enumerate(zip(s1.src, s1.dst))}
    idx = np.array([ref[(int(i) % n, int(j) % n)] for i, j in zip(s2.src, s2.dst)])
    assert np.allclose(s2.y[0].numpy(), s1.y[0].numpy()[idx], atol=1e-6)
    t = structures.tile_structure(structures.Structure(st.z, np.mod(st.pos, L), np.full(3, L)), [2, 1, 3])
    assert np.allclose(t.cell, [2 * L, L, 3 * L]) and np.allclose(t.pos[n * 1:n * 2], np.mod(st.pos, L) + [0, 0, L])
