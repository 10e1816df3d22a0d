"""nablaDFT reader (generated mini database), orbital reordering, label round trip."""
import numpy as np

from maloq_b200.data import readers
from maloq_b200.data.basis_sets import get_basis


def test_reorder_is_a_signed_permutation():
    basis = get_basis("def2_svp_nabla")
    z = [8, 1, 1]
    idx, sgn = readers.reorder_indices(z, basis, "aims")
    assert sorted(idx.tolist()) == list(range(len(idx)))
    H = np.random.default_rng(0).normal(size=(len(idx), len(idx)))
    H2 = readers.reorder_orbitals(H, z, basis, "aims")
    assert np.allclose(np.sort(np.abs(H2).ravel()), np.sort(np.abs(H).ravel()))


def test_nabladft_roundtrip(tmp_path):
    basis = get_basis("def2_svp_nabla")
    rng = np.random.default_rng(1)
    mols = []
    for _ in range(3):
        z = rng.choice([1, 6, 8], size=5).astype(np.int32)
        R = rng.uniform(0, 5, size=(5, 3)) / readers.BOHR_TO_ANGSTROM
        n = sum(sum(2 * l + 1 for l in basis[int(a)]) for a in z)
        H = rng.normal(size=(n, n))
        H = H + H.T
        mols.append((z, R, -1.0, np.zeros((5, 3)), H, np.eye(n), H))
    path = str(tmp_path / "mini.db")
    readers.write_nabladft(path, mols)
    db = readers.NablaDFTDatabase(path)
    assert len(db) == 3
    Z, R, E, F, H, S, C = db[1]
    assert np.allclose(H, mols[1][4].astype(np.float32))
    samples, lab = readers.load_nabladft(path, {"rcut_orbitals": 10.0, "num_structures": 3})
    # labels -> blocks reproduces the reordered Hamiltonian on every stored block
    s = samples[0]
    bsm = lab.blocks_from_labels(s, s.node_y[0], s.y[0])
    dense = bsm.to_dense()
    ref = readers.reorder_orbitals(mols[0][4], mols[0][0], basis, "psi4")
    assert np.allclose(dense, ref, atol=1e-4)
    # energy and forces travel with the sample and collate into batch.energy / batch.forces
    from maloq_b200.data.batch import collate

    assert abs(s.energy - float(np.float32(mols[0][2]))) < 1e-6 and s.forces.shape == (s.num_nodes, 3)
    b = collate(samples, lab.table)
    assert b.energy.shape == (3,) and b.forces.shape == (sum(x.num_nodes for x in samples), 3)


def test_pyscf_orbital_order_up_to_g_shells():
    """PySCF -> e3nn orbital order for s..g shells: p shells permuted (x, y, z) -> (y, z, x) in
    e3nn's (m = -1, 0, 1) order; d shells as they are; f and g shells keep their order with the
    outermost |m| components negated (the reference's PySCF reflections), and the map is the
    inverse of e3nn -> PySCF."""
    import numpy as np

    from maloq_b200.data.readers import reorder_orbitals, reorder_orbitals_inverse

    basis = {8: [0, 1, 2, 3, 4]}
    n = 1 + 3 + 5 + 7 + 9
    rng = np.random.default_rng(0)
    H = rng.standard_normal((n, n))
    H = H + H.T
    He = reorder_orbitals(H, [8], basis, "pyscf")
    assert np.allclose(reorder_orbitals_inverse(He, [8], basis, "pyscf"), H)
    # p block: e3nn row 0 (m=-1) is PySCF row 1, e3nn row 2 (m=+1) is PySCF row 0
    assert np.allclose(He[1:4, 1:4], H[1:4, 1:4][[1, 2, 0]][:, [1, 2, 0]])
    assert np.allclose(He[4:9, 4:9], H[4:9, 4:9])
    sf = np.array([-1, 1, 1, 1, 1, 1, -1.0])
    assert np.allclose(He[9:16, 9:16], H[9:16, 9:16] * np.outer(sf, sf))
    sg = np.array([-1, -1, 1, 1, 1, 1, 1, -1, -1.0])
    assert np.allclose(He[16:, 16:], H[16:, 16:] * np.outer(sg, sg))


def _orca_orbital_text(unrestricted):
    head = ["----------------", "ORBITAL ENERGIES", "----------------", ""]
    tab = lambda e, o: ["  NO   OCC          E(Eh)            E(eV) "] + \
        [f"{i:4d}   {oc:.4f}     {en: .6f}    {en * 27.2114: .4f}" for i, (en, oc) in enumerate(zip(e, o))] + [""]
    if not unrestricted:
        return head + tab([-20.5, -1.3, -0.6, 0.1, 0.4], [2, 2, 2, 0, 0]) + ["", "MULLIKEN POPULATION ANALYSIS", "1 2 3"]
    return head + ["SPIN UP ORBITALS"] + tab([-20.0, -1.0, -0.5, 0.2], [1, 1, 1, 0]) + \
        ["SPIN DOWN ORBITALS"] + tab([-19.9, -0.9, 0.3, 0.5], [1, 1, 0, 0]) + ["", "MULLIKEN POPULATION ANALYSIS"]


def test_orca_orbital_energies_homo_lumo_and_path_conventions(tmp_path):
    import numpy as np

    from maloq_b200.data import readers as R

    eps, occ = R._orbital_energies(_orca_orbital_text(False))
    assert len(eps) == 1 and np.allclose(eps[0], [-20.5, -1.3, -0.6, 0.1, 0.4]) and occ[0].sum() == 6
    assert R.homo_lumo_energies(eps, 6) == ([-0.6], [0.1])
    eps, occ = R._orbital_energies(_orca_orbital_text(True))
    assert len(eps) == 2 and len(eps[1]) == 4
    homo, lumo = R.homo_lumo_energies(eps, 5, multiplicity=2)  # 3 alpha, 2 beta electrons
    assert homo == [-0.5, -0.9] and lumo == [0.2, 0.3]
    d = tmp_path / "mol_17_-1_2" / "step1"
    d.mkdir(parents=True)
    (d / "orca.out").write_text("x")
    assert R.charge_and_multiplicity_from_path(str(d / "orca.out")) == (-1, 2)
    assert R.charge_and_multiplicity_from_path(str(tmp_path / "plain" / "orca.out")) == (0, 1)
    (d / "orca.inp").write_text("%scf\n  FinalMs 0.5\nend\n")
    assert R.read_finalms(str(d / "orca.inp")) == 0.5
    basis = {1: [0, 0, 1], 8: [0, 1, 0, 2, 1]}
    assert R.orbital_count([8, 1, 1], basis) == 1 + 3 + 1 + 5 + 3 + 2 * 5
    H = np.arange(13 * 13, dtype=float).reshape(13, 13)
    Hs = R.sort_by_l(H, basis, [8])
    # O shells s(0) p(1-3) s(4) d(5-9) p(10-12) -> s s p p d
    perm = [0, 4] + [1, 2, 3] + [10, 11, 12] + [5, 6, 7, 8, 9]
    assert np.array_equal(Hs, H[np.ix_(perm, perm)])
