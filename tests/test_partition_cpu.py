"""Graph partitioning: partitioners, decomposition invariants, and partitioned forward/backward
on 2 gloo ranks equal to the single-process result."""
import numpy as np
import pytest
import torch

from maloq_b200.parallel import partition as P
from tests import _dist_util


def _toy_graph(seed=0, n=60):
    from maloq_b200.data import structures
    from maloq_b200.data.batch import make_sample

    rng = np.random.default_rng(seed)
    s = structures.Structure(rng.choice([1, 6, 8], size=n), rng.uniform(0, 9, size=(n, 3)))
    return make_sample(s, 4.0)


@pytest.mark.parametrize("name", sorted(P.PARTITIONERS))
@pytest.mark.parametrize("world", [2, 3, 4])
def test_partitioners_and_decomposition(name, world):
    g = _toy_graph()
    part = P.partition(name, g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    assert part.shape == (g.num_nodes,) and part.min() >= 0 and part.max() < world
    doms = P.decompose(part, g.src, g.dst, world)
    # every edge owned exactly once, by its destination's owner
    all_e = np.sort(np.concatenate([d.edges for d in doms]))
    assert np.array_equal(all_e, np.arange(len(g.src)))
    for d in doms:
        assert np.all(part[g.dst[d.edges]] == d.rank)
        ext = np.concatenate([d.owned, d.halo])
        assert np.array_equal(ext[d.src_local], g.src[d.edges])
        assert np.array_equal(d.owned[d.dst_local], g.dst[d.edges])
        assert np.all(np.diff(d.dst_local) >= 0)
        # the rows each peer sends are exactly that peer's halo block for me
        for p in range(world):
            mine = d.halo[d.halo_owner == p]
            assert np.array_equal(doms[p].owned[doms[p].send[d.rank]], mine)


def _model(lab, edge_chunk=None):
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head

    torch.manual_seed(0)
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=5.0, num_layers=2, num_distance_basis=8,
              edge_channels=8, message_type="source-target-message")
    bb = eSEN_Backbone(lab.irreps, edge_chunk=edge_chunk, edge_stream_dtype=torch.float32, **kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list, reduce_node=True,
                          reduce_node_intra=True)
    return bb, hd


def _partitioned_worker(rank, world, pname, edge_chunk=None):
    import torch.distributed as dist

    from maloq_b200.data import basis_sets
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.parallel.halo import partition_batch

    g = _toy_graph()
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    part = P.partition(pname, g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    dom = P.decompose(part, g.src, g.dst, world)[rank]
    b = partition_batch(g, dom, lab.table)
    bb, hd = _model(lab, edge_chunk)
    no, eo = hd(bb(b), b)
    torch.manual_seed(7)
    wn = torch.randn(g.num_nodes, no.shape[-1])
    we = torch.randn(len(g.src), eo.shape[-1])
    loss = (no[0] * wn[dom.owned]).sum() + (eo[0] * we[dom.edges]).sum()
    loss.backward()
    grads = [p.grad.clone() if p.grad is not None else torch.zeros_like(p) for p in
             list(bb.parameters()) + list(hd.parameters())]
    for gr in grads:
        dist.all_reduce(gr)
    return dom.owned, dom.edges, no[0].detach(), eo[0].detach(), grads


def _single():
    from maloq_b200.data import basis_sets
    from maloq_b200.data.batch import collate
    from maloq_b200.data.targets import FockLabeler

    g = _toy_graph()
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    b = collate([g], lab.table)
    bb, hd = _model(lab)
    no, eo = hd(bb(b), b)
    torch.manual_seed(7)
    wn = torch.randn(g.num_nodes, no.shape[-1])
    we = torch.randn(len(g.src), eo.shape[-1])
    ((no[0] * wn).sum() + (eo[0] * we).sum()).backward()
    return no[0].detach(), eo[0].detach(), [p.grad.clone() if p.grad is not None else torch.zeros_like(p)
                                            for p in list(bb.parameters()) + list(hd.parameters())]


@pytest.mark.parametrize("pname,edge_chunk", [("linear-edgewise", None), ("rcb", None), ("rcb", 40)])
def test_partitioned_forward_backward_matches_single_process(pname, edge_chunk):
    """Graph-partitioned (2 gloo ranks, collective halo) = one process; with ``edge_chunk`` the
    blocks also run over edge chunks sharing one halo exchange per block."""
    ref_n, ref_e, ref_g = _single()
    out = _dist_util.run(_partitioned_worker, world=2, args=(pname, edge_chunk))
    for r, (own, edges, no, eo, grads) in out.items():
        assert np.allclose(no, ref_n[own].numpy(), atol=1e-5, rtol=1e-4)
        assert np.allclose(eo, ref_e[edges].numpy(), atol=1e-5, rtol=1e-4)
        for a, b in zip(grads, ref_g):
            assert np.allclose(a, b.numpy(), atol=1e-4, rtol=1e-3)


def _workflow_worker(rank, world, folder, mode):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_sio2", num_atoms=150, distribute_graphs=True, partition_type="slab",
               l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.0, rcut_gaussian=4.0,
               mmax=2, num_epochs=2, lr_init=1e-3, device="cpu", output_folder=folder, train_or_eval=mode,
               log_every=0, save_frequency=1)
    return training_workflow.TrainingWorkflow(cfg).run()


def test_partitioned_workflow_train_and_infer(tmp_path):
    out = _dist_util.run(_workflow_worker, world=2, args=(str(tmp_path), "train"))
    hist = out[0]
    assert len(hist["train_node"]) == 2 and np.isfinite(hist["train_node"]).all()
    _dist_util.run(_workflow_worker, world=2, args=(str(tmp_path), "infer"))
    from maloq_b200.data import datasets
    from maloq_b200.parallel.infer import load_partitioned_hamiltonian

    H = load_partitioned_hamiltonian(str(tmp_path), datasets.labeler_for("sio2"))
    dense = H.to_dense()
    assert dense.shape[0] == 150 * 13
    assert np.allclose(dense, dense.T, atol=1e-5)
    import scipy.sparse as sp

    path = H.save_npz(str(tmp_path / "H.npz"))
    assert np.allclose(sp.load_npz(path).toarray(), dense)


def _local_domain_worker(rank, world):
    import torch

    g = _toy_graph(seed=3, n=80)
    part = P.partition("slab", g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    ref = P.decompose(part, g.src, g.dst, world)[rank]
    # this rank's edges as a per-rank builder produces them: into owned atoms, (dst row, src) order
    sel = ref.edges
    dom, src_local = P.local_domain(part, rank, world, torch.as_tensor(g.src[sel]))
    return (ref.owned, dom.owned, ref.halo, dom.halo, ref.halo_owner, dom.halo_owner, ref.halo_row, dom.halo_row,
            ref.src_local, src_local.numpy(), ref.recv_counts, dom.recv_counts,
            [np.asarray(x) for x in ref.send], [np.asarray(x) for x in dom.send])


def test_local_domain_matches_global_decomposition():
    """A domain built from one rank's own edges (no global edge list) equals the one cut from
    the global graph: owned rows, halo order, owners, rows, edge sources and send lists."""
    out = _dist_util.run(_local_domain_worker, world=2)
    for r, v in out.items():
        for a, b in zip(v[0:10:2], v[1:10:2]):
            assert np.array_equal(np.asarray(a), np.asarray(b)), r
        assert list(v[10]) == list(v[11])
        for a, b in zip(v[12], v[13]):
            assert np.array_equal(a, b)


def test_graph_aware_bisections_keep_halo_small():
    g = _toy_graph(seed=5, n=200)
    hv = {name: P.halo_volume(P.partition(name, g.num_nodes, 4, src=g.src, dst=g.dst, pos=g.pos), g.src, g.dst)
          for name in ["rcb", "surface_volume", "approx_neighbors", "local_optimal", "bruteforce", "worst-case"]}
    # the exhaustive search over per-level axis sequences beats each single-axis bisection
    deg = np.bincount(g.dst, minlength=g.num_nodes) + 1
    for ax in range(3):
        fixed = P._bisect(g.num_nodes, 4, g.pos, deg, lambda idx, per, k, ax=ax: ax, [False] * 3)
        assert hv["bruteforce"] <= P.halo_volume(fixed, g.src, g.dst)
    assert hv["bruteforce"] <= 1.1 * min(hv["rcb"], hv["surface_volume"], hv["approx_neighbors"])
    assert hv["local_optimal"] < hv["worst-case"] and hv["bruteforce"] < 0.7 * hv["worst-case"]


def _cp2k_worker(rank, world, data, folder):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="cp2k", dbpath=data, distribute_graphs=True, partition_type="linear-edgewise",
               l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, rcut_orbitals=3.0, rcut_gaussian=6.0,
               mmax=2, num_epochs=2, lr_init=1e-3, device="cpu", output_folder=folder, log_every=0, edge_chunk=500)
    return training_workflow.TrainingWorkflow(cfg).run()


def test_partitioned_workflow_on_a_cp2k_structure(tmp_path):
    """dataset cp2k + distribute_graphs: every rank reads the structure and the dumped
    Hamiltonian, keeps its domain's targets, and trains (chunked blocks, 2 gloo ranks)."""
    import scipy.sparse as sp

    from maloq_b200.data import readers, structures

    rng = np.random.default_rng(7)
    st = structures.amorphous_sio2(rng, 90)
    d = tmp_path / "data" / "s0"
    d.mkdir(parents=True)
    sym = {14: "Si", 8: "O"}
    lines = [str(len(st.z)), "Cell: 13 13 13"] + [f"{sym[int(z)]} {p[0]:.6f} {p[1]:.6f} {p[2]:.6f}"
                                                 for z, p in zip(st.z, np.mod(st.pos * 13.0 / st.cell, 13.0))]
    (d / "structure.xyz").write_text("\n".join(lines) + "\n")
    n = 13 * len(st.z)
    A = sp.random(n, n, density=0.02, random_state=0)
    readers.write_cp2k_csr(d / "hamiltonian.csr", (A + A.T).tocsr())
    out = _dist_util.run(_cp2k_worker, world=2, args=(str(tmp_path / "data"), str(tmp_path / "out")))
    assert len(out[0]["train_node"]) == 2 and np.isfinite(out[0]["train_node"]).all()


def _stream_infer_worker(rank, world):
    import torch

    from maloq_b200.data import datasets, structures
    from maloq_b200.data.graph import radius_graph
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel import partition as P
    from maloq_b200.parallel.halo import local_batch
    from maloq_b200.parallel.infer import hamiltonian_shard

    rng = np.random.default_rng(3)
    st = structures.si_slab_with_oxide(rng, 700)
    lab = datasets.labeler_for("slab")
    part = P.partition("slab", len(st.z), world, pos=st.pos, cell=st.cell)
    owned = np.flatnonzero(part == rank)
    src, dst, vec = radius_graph(st.pos, 6.0, st.cell)
    keep = np.isin(dst, owned)  # the edges into my atoms, (owned row, src) order
    row = np.full(len(st.z), -1)
    row[owned] = np.arange(len(owned))
    s, d, v = src[keep], row[dst[keep]], vec[keep]
    o = np.lexsort((s, d))
    s, d, v = torch.as_tensor(s[o]), torch.as_tensor(d[o]), torch.as_tensor(v[o])
    ptr = torch.zeros(len(owned) + 1, dtype=torch.long)
    ptr[1:] = torch.cumsum(torch.bincount(d, minlength=len(owned)), 0)
    dom, src_local = P.local_domain(part, rank, world, s)
    b = local_batch(st.z, st.pos, dom, src_local, d, v, ptr, lab.table, device="cpu", transport="collective")
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=6.0, edge_channels=8, num_layers=2,
              num_distance_basis=8, edge_stream_dtype=torch.float32)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, edge_chunk=300, **kw).eval()
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True).eval()
    with torch.no_grad():
        data, bptr = hamiltonian_shard(hd, bb(b), b, lab)
    gsrc = np.concatenate([dom.owned, dom.halo])[src_local.numpy()]
    return owned, gsrc, dom.owned[d.numpy()], data.numpy(), bptr.numpy()


def test_streamed_partitioned_inference_matches_single_process():
    """Per-rank edges -> local_domain -> local_batch -> chunked streaming inference (collective
    halo) -> Hamiltonian shard: every block equals the unpartitioned model's block."""
    import torch

    from maloq_b200.data import datasets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel.infer import hamiltonian_shard

    out = _dist_util.run(_stream_infer_worker, world=2)
    rng = np.random.default_rng(3)
    st = structures.si_slab_with_oxide(rng, 700)
    lab = datasets.labeler_for("slab")
    smp = make_sample(st, 6.0)
    b = collate([smp], lab.table)
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=6.0, edge_channels=8, num_layers=2,
              num_distance_basis=8)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, **kw).eval()
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True).eval()
    with torch.no_grad():
        ref, rptr = hamiltonian_shard(hd, bb(b), b, lab)
    ref, rptr = ref.numpy(), rptr.numpy()
    E = len(smp.src)
    key = {(int(a), int(c)): i for i, (a, c) in enumerate(zip(smp.src, smp.dst))}
    n_checked = 0
    for owned, gsrc, gdst, data, bptr in out.values():
        for j, (a, c) in enumerate(zip(gsrc, gdst)):
            i = key[(int(a), int(c))]
            assert np.allclose(data[bptr[j]:bptr[j + 1]], ref[rptr[i]:rptr[i + 1]], atol=2e-4), (a, c)
            n_checked += 1
        ne = len(gsrc)
        for j, a in enumerate(owned):  # on-site blocks follow the edge blocks
            assert np.allclose(data[bptr[ne + j]:bptr[ne + j + 1]], ref[rptr[E + a]:rptr[E + a + 1]], atol=2e-4)
    assert n_checked == E


def test_multilevel_partitioner_beats_greedy_and_balances():
    """``metis`` (multilevel k-way) cuts fewer halo rows than region growing on a periodic
    amorphous cell, keeps the edge load within a few percent, and finds the straight cut of a
    grid graph."""
    from maloq_b200.data import datasets
    from maloq_b200.parallel import partition as P

    s = datasets.build_samples("sio2", 1, seed=0, n_atoms=1500, cutoff=5.0)[0]
    for k in (2, 4):
        pm = P.partition("metis", s.num_nodes, k, src=s.src, dst=s.dst)
        pg = P.partition("greedy", s.num_nodes, k, src=s.src, dst=s.dst)
        assert P.halo_volume(pm, s.src, s.dst) < P.halo_volume(pg, s.src, s.dst)
        assert (pm[s.src] != pm[s.dst]).sum() < (pg[s.src] != pg[s.dst]).sum()
        load = np.bincount(pm, weights=np.bincount(s.dst, minlength=s.num_nodes) + 1.0, minlength=k)
        assert load.max() / load.mean() < 1.06
    # 40 x 10 grid: the best bisection cuts 10 edges (a straight cut across the short side)
    nx, ny = 40, 10
    idx = np.arange(nx * ny).reshape(nx, ny)
    a = np.concatenate([idx[:-1].ravel(), idx[:, :-1].ravel()])
    b = np.concatenate([idx[1:].ravel(), idx[:, 1:].ravel()])
    src, dst = np.concatenate([a, b]), np.concatenate([b, a])
    part = P.partition("metis", nx * ny, 2, src=src, dst=dst)
    cut_pairs = int((part[a] != part[b]).sum())
    assert cut_pairs <= 14, cut_pairs


def _molecule_batches_worker(rank, world, folder, mode):
    from maloq_b200.train.workflow import TrainingWorkflow

    cfg = dict(dataset_name="synthetic_small", num_structures=10, num_train=7, num_val=3, batch_size=2,
               distribute_graphs=True, partition_type="rcb", l_embedding_dim=8, num_mp_layers=1,
               num_distance_basis=8, mmax=2, num_epochs=2, lr_init=1e-3, device="cpu", output_folder=folder,
               log_every=0, save_frequency=0, train_or_eval=mode)
    wf = TrainingWorkflow(cfg)
    train, val, _ = wf.prepare_data()
    cover = [(b.global_node_ids.numpy(), b.atom_mol_id.numpy(), b.node_y.numpy()) for b in train]
    hist = wf.run() if mode == "train" else None
    return len(train), len(val), cover, hist["train_node"] if hist else None


@pytest.mark.parametrize("mode", ["train", "eval"])
def test_distribute_graphs_over_molecule_batches(tmp_path, mode):
    """distribute_graphs on a molecule dataset: batches of molecules become one disjoint-union
    graph each, split over both ranks.  Training: supergraph i joins molecules
    [2i, 2i+2) of every rank's share; evaluation: the ranks take turns broadcasting their share.
    Together the ranks own every atom of every supergraph exactly once, with its targets, and
    training runs."""
    from maloq_b200.data import batch as B
    from maloq_b200.train.workflow import TrainingWorkflow

    out = _dist_util.run(_molecule_batches_worker, world=2, args=(str(tmp_path), mode))
    wf = TrainingWorkflow(dict(dataset_name="synthetic_small", num_structures=10, l_embedding_dim=8,
                               num_mp_layers=1, num_distance_basis=8, mmax=2, device="cpu",
                               output_folder=str(tmp_path)))
    samples, _ = wf._load_global_samples(wf.config)
    share = [samples[0:4], samples[4:7]]  # 7 training molecules: 4 on rank 0, 3 on rank 1
    if mode == "train":
        groups = [share[0][0:2] + share[1][0:2], share[0][2:4] + share[1][2:3]]
    else:
        groups = [share[0][0:2], share[0][2:4], share[1][0:2], share[1][2:3]]
    assert out[0][0] == out[1][0] == len(groups)
    assert out[0][1] == out[1][1] == (1 if mode == "train" else 2)  # 3 val molecules: 2 + 1
    for k, grp in enumerate(groups):
        g = B.merge_samples(grp)
        ids = np.concatenate([out[r][2][k][0] for r in (0, 1)])
        assert np.array_equal(np.sort(ids), np.arange(g.num_nodes))
        for r in (0, 1):
            own, mol, ny = out[r][2][k]
            assert np.array_equal(mol, g.atom_mol_id[own])
            assert np.allclose(ny, g.node_y[:, own].numpy())
    if mode == "train":
        for r in (0, 1):
            assert len(out[r][3]) == 2 and np.isfinite(out[r][3]).all()


def _molecule_eval_worker(rank, world, folder, mode):
    from maloq_b200.train.workflow import TrainingWorkflow

    cfg = dict(dataset_name="synthetic_small", num_structures=10, num_train=7, num_val=3, batch_size=1,
               partition_type="rcb", l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, mmax=2,
               num_epochs=1, lr_init=1e-3, device="cpu", output_folder=folder, log_every=0, save_frequency=1,
               distribute_graphs=True, train_or_eval=mode)
    if mode == "eval":
        cfg.update(restart_backbone=True, restart_head=True)
    return TrainingWorkflow(cfg).run()


def test_partitioned_molecule_evaluation_matches_single_process(tmp_path):
    """Evaluation with distribute_graphs on molecules: each validation molecule is split over two
    ranks, the outputs are gathered to rank 0 and cut back into molecules; the per-molecule
    errors equal those of an unpartitioned evaluation of the same checkpoint."""
    from maloq_b200.train.workflow import TrainingWorkflow

    _dist_util.run(_molecule_eval_worker, world=2, args=(str(tmp_path), "train"))
    out = _dist_util.run(_molecule_eval_worker, world=2, args=(str(tmp_path), "eval"))
    rows = out[0]
    assert len(rows) == 3 and out[1] == []
    single = TrainingWorkflow(dict(dataset_name="synthetic_small", num_structures=10, num_train=7, num_val=3,
                                   batch_size=1, l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, mmax=2,
                                   device="cpu", output_folder=str(tmp_path), train_or_eval="eval",
                                   restart_backbone=True, restart_head=True, log_every=0)).run()
    assert len(single) == 3
    for a, b in zip(rows, single):
        assert a[0] == b[0] and a[-1] == b[-1]
        np.testing.assert_allclose(np.array(a[1:-1], dtype=float), np.array(b[1:-1], dtype=float),
                                   rtol=1e-4, atol=1e-6)


def test_source_csr_offsets():
    """The source-grouped CSR of the edge kernels' backward (perm, ptr) from a sorted search:
    ptr[i] counts edges with source < i, including sources with no edges and halo rows."""
    import torch

    from maloq_b200.ops.edge_native import src_csr

    class G:
        pass

    rng = np.random.default_rng(0)
    g = G()
    g.src = torch.as_tensor(rng.integers(0, 40, size=500))
    g.src[g.src == 7] = 8  # a node without outgoing edges
    g.num_nodes, g.num_nodes_ext, g.cache = 38, 45, {}
    perm, ptr = src_csr(g)
    assert ptr.shape == (46,) and ptr.dtype == torch.long
    ref = np.concatenate([[0], np.cumsum(np.bincount(g.src.numpy(), minlength=45))])
    assert np.array_equal(ptr.numpy(), ref)
    assert np.array_equal(g.src[perm].numpy(), np.sort(g.src.numpy(), kind="stable"))


def _partitioned_kernel_path_worker(rank, world, pname, edge_chunk):
    """The partitioned worker with the kernel path on the CPU stand-in of the extension."""
    from maloq_b200 import ops
    from maloq_b200.ops import kernels
    from maloq_b200.ops import loss as ops_loss
    from tests.cpu_extension import CpuExtension

    kernels._lib = CpuExtension()
    ops._cuda = ops_loss._cuda = lambda *t: True
    return _partitioned_worker(rank, world, pname, edge_chunk)


@pytest.mark.parametrize("pname,edge_chunk", [("rcb", None), ("linear-edgewise", 40)])
def test_partitioned_kernel_path_matches_single_process(monkeypatch, pname, edge_chunk):
    """Graph partitioned over 2 gloo ranks (collective halo) on the kernel path = one process on
    the kernel path (both on the CPU stand-in of the extension: the same bf16 roundings, so the
    partitioned exchange must reproduce the single-process values closely)."""
    from tests.cpu_extension import use_cpu_extension

    out = _dist_util.run(_partitioned_kernel_path_worker, world=2, args=(pname, edge_chunk))
    use_cpu_extension(monkeypatch)
    ref_n, ref_e, ref_g = _single()
    rel = lambda a, b: float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-12))
    for r, (own, edges, no, eo, grads) in out.items():
        assert rel(no, ref_n[own].numpy()) < 2e-3
        assert rel(eo, ref_e[edges].numpy()) < 2e-3
        worst = max(rel(a, b.numpy()) for a, b in zip(grads, ref_g) if np.linalg.norm(b.numpy()) > 0)
        assert worst < 1e-2, worst


@pytest.mark.parametrize("pname,world", [("slab", 4), ("rcb", 8), ("linear-edgewise", 3)])
def test_halo_neighbour_sets_are_symmetric(pname, world):
    """The NVLink halo's peer barriers include only halo neighbours; that is safe only if the
    neighbour relation is symmetric (a rank waits on exactly the ranks that signal it)."""
    from maloq_b200.parallel.peer_halo import halo_neighbours

    g = _toy_graph(seed=5, n=200)
    part = P.partition(pname, g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    doms = P.decompose(part, g.src, g.dst, world)
    nb = [set(halo_neighbours(d)) for d in doms]
    for r in range(world):
        assert r not in nb[r]
        for p in nb[r]:
            assert r in nb[p]
        # every rank whose rows r reads is a neighbour
        assert {int(o) for o in doms[r].halo_owner} <= nb[r]


def _peer_halo_worker(rank, world, folder, pname, edge_chunk):
    """The partitioned worker on the NVLink halo transport, with symmetric memory emulated in
    host shared memory and the kernel path on the CPU stand-in."""
    import torch.distributed as dist

    from maloq_b200 import ops
    from maloq_b200.data import basis_sets
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.ops import kernels
    from maloq_b200.ops import loss as ops_loss
    from maloq_b200.parallel.halo import partition_batch
    from tests import fake_symm
    from tests.cpu_extension import CpuExtension

    fake_symm.install(folder)
    kernels._lib = CpuExtension()
    ops._cuda = ops_loss._cuda = lambda *t: True
    g = _toy_graph()
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    part = P.partition(pname, g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    dom = P.decompose(part, g.src, g.dst, world)[rank]
    b = partition_batch(g, dom, lab.table, transport="peer")
    bb, hd = _model(lab, edge_chunk)
    no, eo = hd(bb(b), b)
    torch.manual_seed(7)
    wn = torch.randn(g.num_nodes, no.shape[-1])
    we = torch.randn(len(g.src), eo.shape[-1])
    loss = (no[0] * wn[dom.owned]).sum() + (eo[0] * we[dom.edges]).sum()
    loss.backward()
    grads = [p.grad.clone() if p.grad is not None else torch.zeros_like(p) for p in
             list(bb.parameters()) + list(hd.parameters())]
    for gr in grads:
        dist.all_reduce(gr)
    peer = b.halo.peer
    return (dom.owned, dom.edges, no[0].detach(), eo[0].detach(), grads, kernels._lib.error_status(True),
            None if peer is None else (peer.neighbours, peer.epoch))


@pytest.mark.parametrize("pname,world,edge_chunk", [("slab", 2, None), ("slab", 3, None), ("rcb", 3, 40)])
def test_nvlink_halo_path_on_emulated_peer_memory(monkeypatch, tmp_path, pname, world, edge_chunk):
    """The NVLink halo transport (publish to staging slots, neighbour barriers, halo rows read
    from the owners' memory inside the gather, halo gradients pushed to the owners and summed
    there) on symmetric memory emulated in shared memory across gloo processes: equal to the
    single-process kernel path, no barrier timed out, and each rank's barriers include only its
    halo neighbours."""
    from tests.cpu_extension import use_cpu_extension

    out = _dist_util.run(_peer_halo_worker, world=world, args=(str(tmp_path), pname, edge_chunk), timeout=300)
    use_cpu_extension(monkeypatch)
    ref_n, ref_e, ref_g = _single()
    rel = lambda a, b: float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-12))
    for r, (own, edges, no, eo, grads, err, peer) in out.items():
        assert err == 0
        assert rel(no, ref_n[own].numpy()) < 2e-3 and rel(eo, ref_e[edges].numpy()) < 2e-3
        worst = max(rel(a, b.numpy()) for a, b in zip(grads, ref_g) if np.linalg.norm(b.numpy()) > 0)
        assert worst < 1e-2, worst
        assert peer is not None and peer[1] > 0 and r not in peer[0]


def _peer_workflow_worker(rank, world, folder, transport):
    from maloq_b200 import ops
    from maloq_b200.ops import basis_transform, kernels, labels
    from maloq_b200.ops import loss as ops_loss
    from maloq_b200.train.workflow import TrainingWorkflow
    from tests import fake_symm
    from tests.cpu_extension import CpuExtension

    fake_symm.install(folder + "/symm")
    kernels._lib = CpuExtension()
    for m in (ops, ops_loss, labels, basis_transform):
        m._cuda = lambda *t: True
    cfg = dict(dataset_name="synthetic_sio2", num_atoms=90, distribute_graphs=True, partition_type="slab",
               halo_transport=transport, l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8,
               rcut_orbitals=2.0, rcut_gaussian=4.0, mmax=2, num_epochs=2, lr_init=1e-3, device="cpu",
               output_folder=folder + "/" + transport, log_every=0, save_frequency=0)
    hist = TrainingWorkflow(cfg).run()
    return hist["train_node"], hist["train_edge"], kernels._lib.error_status(True)


def test_partitioned_training_on_the_nvlink_halo_transport(tmp_path):
    """Two epochs of graph-partitioned training (3 ranks, slab partition) on the kernel path:
    the NVLink halo transport on emulated peer memory (staging slots and receive buffers reused
    across layers and steps) gives the same losses as the collective transport."""
    runs = {t: _dist_util.run(_peer_workflow_worker, world=3, args=(str(tmp_path), t), timeout=600)
            for t in ("peer", "collective")}
    for r in range(3):
        pn, pe, err = runs["peer"][r]
        cn, ce, _ = runs["collective"][r]
        assert err == 0
        assert np.allclose(pn, cn, rtol=1e-4) and np.allclose(pe, ce, rtol=1e-4), (pn, cn)
