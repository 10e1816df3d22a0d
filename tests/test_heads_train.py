"""Heads (reduce_edge, open shell, energy, forces), checkpoint resume, optimizers."""
import numpy as np
import pytest
import torch

from maloq_b200.core import sph
from maloq_b200.data import basis_sets, structures
from maloq_b200.data.batch import collate, make_sample
from maloq_b200.data.targets import FockLabeler
from maloq_b200.models.backbone import eSEN_Backbone
from maloq_b200.models.heads import Fock_Irreps_Head, HELM_Energy_Head, HELM_Force_Head

P = np.array([[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])
KW = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=5.0, num_layers=2, num_distance_basis=8,
          edge_channels=8)


def _batches(R_in, dtype=torch.float64, include_edges=True):
    rng = np.random.default_rng(3)
    structs = [structures.random_small_molecule(rng) for _ in range(2)]
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"), dtype=dtype)
    out = [make_sample(structures.Structure(s.z, s.pos @ R_in.T), 5.0) for s in structs]
    return collate(out, lab.table, float_dtype=dtype), lab


def test_reduce_edge_head_equivariant_and_symmetric():
    R_in = sph.euler_matrix(0.3, 1.2, -0.5)
    Dm = P @ R_in @ P.T
    b0, lab = _batches(np.eye(3))
    b1, _ = _batches(R_in)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, **KW).double()
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list, reduce_node=True,
                          reduce_node_intra=True, reduce_edge=True).double()
    n0, e0 = hd(bb(b0), b0)
    n1, e1 = hd(bb(b1), b1)
    Dl = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(it.l, Dm)) for it in lab.irreps])
    assert (e0[0] @ Dl.T - e1[0]).abs().max() < 1e-8
    assert (n0[0] @ Dl.T - n1[0]).abs().max() < 1e-8
    # the reconstructed (i,j) and (j,i) blocks are transposes of each other
    s = b0
    blocks = lab.blocks_from_labels(_sample_of(s, 0, lab), n0[0][: int(s.num_atoms_in_molecule[0])],
                                    e0[0][: _n_edges(s, 0)])
    H = blocks.to_dense()
    assert np.allclose(H, H.T, atol=1e-8)


def _n_edges(b, g):
    nat = b.num_atoms_in_molecule.tolist()
    dst = b.edge_index[1].numpy()
    return int((dst < nat[0]).sum()) if g == 0 else None


def _sample_of(b, g, lab):
    from maloq_b200.data.batch import GraphSample

    n = int(b.num_atoms_in_molecule[0])
    ne = _n_edges(b, 0)
    ei = b.edge_index[:, :ne].numpy()
    return GraphSample(b.atomic_numbers[:n].numpy(), b.pos[:n].numpy(), ei[0], ei[1], b.edge_attr[:ne].numpy())


def test_open_shell_head_outputs_two_spins():
    b, lab = _batches(np.eye(3), torch.float32)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, open_shell=True, **KW)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list, open_shell=True,
                          reduce_node=True, reduce_node_intra=True)
    n, e = hd(bb(b), b)
    assert n.shape[0] == 2 and e.shape[0] == 2 and not torch.allclose(n[0], n[1])


def test_energy_invariant_and_forces_equivariant():
    R_in = sph.euler_matrix(-0.7, 0.4, 2.0)
    Rm = P @ R_in @ P.T
    b0, lab = _batches(np.eye(3))
    b1, _ = _batches(R_in)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, include_edges=False, **KW).double()
    eh = HELM_Energy_Head(bb).double()
    fh = HELM_Force_Head(bb).double()
    e0, e1 = eh(bb(b0), b0)["energies"], eh(bb(b1), b1)["energies"]
    assert e0.shape == (2,) and torch.allclose(e0, e1, atol=1e-9)
    f0, f1 = fh(bb(b0), b0)["forces"], fh(bb(b1), b1)["forces"]
    D1 = torch.tensor(sph.wigner_D_from_matrix(1, Rm))
    assert torch.allclose(f0 @ D1.T, f1, atol=1e-9)


def test_checkpoint_resume_continues(tmp_path):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=12, batch_size=6, num_epochs=2, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", save_frequency=1, log_every=0)
    h1 = training_workflow.TrainingWorkflow(cfg).run()
    sd1 = torch.load(tmp_path / "backbone.pt", weights_only=False)["model_state_dict"]
    cfg2 = dict(cfg, num_epochs=3, restart_backbone=True, restart_head=True, restart_optimizer=True)
    h2 = training_workflow.TrainingWorkflow(cfg2).run()
    assert len(h2["train_node"]) == 3 and h2["train_node"][:2] == h1["train_node"]
    sd2 = torch.load(tmp_path / "backbone.pt", weights_only=False)["model_state_dict"]
    assert any(not torch.equal(sd1[k], sd2[k]) for k in sd1 if sd1[k].is_floating_point())


@pytest.mark.parametrize("opt", ["adam", "adamw", "muon"])
def test_optimizers_reduce_loss(tmp_path, opt):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=10, batch_size=5, num_epochs=4, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2, lr_init=3e-3,
               muon_lr=0.01, optimizer_type=opt, output_folder=str(tmp_path), device="cpu", log_every=0,
               scheduler_type="plateau")
    h = training_workflow.TrainingWorkflow(cfg).run()
    assert h["train_node"][-1] < h["train_node"][0]


def test_state_dict_keys_follow_reference_layout():
    _, lab = _batches(np.eye(3), torch.float32)
    bb = eSEN_Backbone(lab.irreps, **KW)
    keys = set(bb.state_dict())
    for k in ["Jd_0", "Jd_4", "distance_expansion.offset", "sphere_embedding.weight", "scalar_node_embedding.bias",
              "edge_degree_embedding.rad_func.net.6.weight", "node_blocks.0.norm_1.affine_weight",
              "node_blocks.0.norm_1.balance_degree_weight", "node_blocks.0.edge_wise.act.expand_index",
              "node_blocks.0.edge_wise.so2_conv_1.fc_m0.weight", "node_blocks.0.edge_wise.so2_conv_1.so2_m_conv.1.fc.weight",
              "node_blocks.0.edge_wise.so2_conv_1.rad_func.net.4.bias", "node_blocks.1.atom_wise.so3_linear_2.expand_index",
              "edge_blocks.1.atom_wise.scalar_mlp.0.weight", "norm.affine_bias"]:
        assert k in keys, k
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list, reduce_node=True,
                          reduce_node_intra=True)
    hk = set(hd.state_dict())
    for k in ["parity_multiplier", "lin_scalars_learnable.0.weight", "node_lin_out_layers.0.2.weight",
              "edge_lin_out_layers.0.4.weight"]:
        assert k in hk, k


def test_activation_checkpointing_matches_plain_backward():
    b, lab = _batches(np.eye(3))
    grads = []
    for ckpt in (False, True):
        torch.manual_seed(0)
        bb = eSEN_Backbone(lab.irreps, activation_checkpointing=ckpt, **KW).double()
        out = bb(b)
        loss = out["node_embeddings"].pow(2).sum() + out["edge_embeddings"].pow(2).sum()
        loss.backward()
        grads.append([p.grad.clone() for p in bb.parameters()])
    for g0, g1 in zip(*grads):
        assert torch.allclose(g0, g1, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("chunk,stream", [(7, "fp64"), (25, "fp64"), (7, "bf16")])
def test_edge_chunked_execution_matches_unchunked(chunk, stream):
    """Chunked blocks (whole destination nodes per chunk, recomputed in backward) give the
    unchunked forward and gradients: exactly with a full-precision edge stream, and up to the
    bf16 rounding of the stored edge stream otherwise."""
    dtype = torch.float64 if stream == "fp64" else torch.float32
    b, lab = _batches(np.eye(3), dtype=dtype)
    sd = torch.float64 if stream == "fp64" else torch.bfloat16
    res = []
    for ec in (None, chunk):
        torch.manual_seed(0)
        bb = eSEN_Backbone(lab.irreps, edge_chunk=ec, edge_stream_dtype=sd, **KW).to(dtype)
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                              reduce_node=True, reduce_node_intra=True).to(dtype)
        emb = bb(b)
        if ec is not None:
            assert emb.get("edge_chunks") and len(emb["edge_chunks"]) > 1
        n, e = hd(emb, b)
        (n.pow(2).sum() + e.pow(2).sum()).backward()
        params = list(bb.parameters()) + list(hd.parameters())
        res.append((n.detach(), e.detach(), [torch.zeros_like(p) if p.grad is None else p.grad.clone() for p in params]))
    (n0, e0, g0), (n1, e1, g1) = res
    if stream == "fp64":
        assert torch.allclose(n0, n1, rtol=1e-10, atol=1e-12)
        assert torch.allclose(e0, e1, rtol=1e-10, atol=1e-12)
        for a, c in zip(g0, g1):
            assert torch.allclose(a, c, rtol=1e-9, atol=1e-11)
        return
    for x, y in ((n0, n1), (e0, e1)):
        assert (x - y).abs().max() <= 2e-2 * x.abs().max()
    for a, c in zip(g0, g1):
        if a.numel():
            assert (a - c).abs().max() <= 5e-2 * max(1e-6, a.abs().max().item())


def test_chunked_inference_streams_in_place_and_matches():
    """Without gradients the chunked forward overwrites the edge stream in place and computes
    each chunk's rotations on use; it equals the unchunked forward."""
    b, lab = _batches(np.eye(3), dtype=torch.float64)
    outs = []
    for ec in (None, 9):
        torch.manual_seed(0)
        bb = eSEN_Backbone(lab.irreps, edge_chunk=ec, edge_stream_dtype=torch.float64, **KW).double()
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                              reduce_node=True, reduce_node_intra=True).double()
        with torch.no_grad():
            g = bb.build_graph(b)
            if ec is not None:
                assert g.rot is None and g.rot_fn is not None and len(g.chunks) > 1
            emb = bb(b)
            outs.append(hd(emb, b))
    (n0, e0), (n1, e1) = outs
    assert torch.allclose(n0, n1, rtol=1e-10, atol=1e-12)
    assert torch.allclose(e0, e1, rtol=1e-10, atol=1e-12)


def test_streamed_hamiltonian_shard_matches_full_conversion():
    from maloq_b200.ops import labels as lab_ops
    from maloq_b200.parallel.infer import hamiltonian_shard

    b, lab = _batches(np.eye(3), dtype=torch.float64)
    tbl = lab.table
    b.edge_pair_type = torch.as_tensor(tbl.pair_type(b.src_z.numpy(), b.dst_z.numpy()))
    b.node_pair_type = torch.as_tensor(tbl.pair_type(b.atomic_numbers.numpy(), b.atomic_numbers.numpy()))
    res = []
    for ec in (None, 9):
        torch.manual_seed(0)
        bb = eSEN_Backbone(lab.irreps, edge_chunk=ec, edge_stream_dtype=torch.float64, **KW).double()
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                              reduce_node=True, reduce_node_intra=True).double()
        with torch.no_grad():
            emb = bb(b)
            if ec is None:
                no, eo = hd(emb, b)
                data, ptr = hamiltonian_shard(hd, emb, b, lab)
                full = lab_ops.coupled_to_blocks(torch.cat([eo[0], no[0]]), ptr,
                                                 torch.cat([b.edge_pair_type, b.node_pair_type]), lab.pos_t,
                                                 lab.transform, int(ptr[-1]))
                assert torch.allclose(data.double(), full.double(), atol=1e-10)
            else:
                data, ptr = hamiltonian_shard(hd, emb, b, lab)
        res.append(data)
    assert torch.allclose(res[0].double(), res[1].double(), atol=1e-10)


@pytest.mark.parametrize("target", ["energies", "forces"])
def test_workflow_trains_energy_and_force_targets(tmp_path, target):
    """loss_target energies / forces: teacher targets on the samples, the HELM energy / force
    head, and a loss that goes down."""
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=12, batch_size=4, num_epochs=5, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2, lr_init=3e-3,
               loss_target=target, output_folder=str(tmp_path), device="cpu", log_every=0)
    h = training_workflow.TrainingWorkflow(cfg).run()
    assert np.isfinite(h["train_node"][-1]) and h["train_node"][-1] < h["train_node"][0]


def test_scale_shift_and_uncoupled_loss_in_workflow(tmp_path):
    """scale_and_shift writes the per-element l=0 table (reference key names) and the
    shifted targets have zero per-element mean; compute_uncoupled_loss trains through the
    differentiable basis transform; evaluation un-shifts."""
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=12, batch_size=4, num_epochs=3, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2, lr_init=3e-3,
               scale_and_shift=True, compute_uncoupled_loss=True, output_folder=str(tmp_path), device="cpu",
               log_every=0)
    wf = training_workflow.TrainingWorkflow(cfg)
    h = wf.run()
    assert h["train_node"][-1] < h["train_node"][0]
    d = torch.load(tmp_path / "element_scale_shifts_synthetic_small.pt", weights_only=False)
    assert set(d) == {"element_scalar_means", "element_scalar_stds", "scalar_irrep_indices"}
    ev = training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True,
                                                 restart_head=True)).run()
    assert np.isfinite(ev[0][1])


def test_energy_linear_references(tmp_path):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=12, batch_size=4, num_epochs=2, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               loss_target="energies", scale_and_shift=True, output_folder=str(tmp_path), device="cpu", log_every=0)
    wf = training_workflow.TrainingWorkflow(cfg)
    wf.run()
    coeff = np.load(tmp_path / "lin_ref_coeffs_synthetic_small.npz")["coeff"]
    assert coeff.ndim == 1 and np.isfinite(coeff).all() and wf.energy_refs is not None


@pytest.mark.parametrize("extra", [dict(open_shell=True), dict(reduce_edge=True),
                                   dict(message_type="source-target-message")])
def test_workflow_variants_train(tmp_path, extra):
    """Open shell (alpha/beta teacher targets), reduce_edge and the 3-way message all train."""
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=8, batch_size=4, num_epochs=2, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               output_folder=str(tmp_path), device="cpu", log_every=0, **extra)
    h = training_workflow.TrainingWorkflow(cfg).run()
    assert len(h["train_node"]) == 2 and np.isfinite(h["train_node"]).all()


@pytest.mark.parametrize("target", ["energies", "forces"])
def test_workflow_eval_energy_and_force_heads(tmp_path, target):
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=8, batch_size=4, num_epochs=1, l_embedding_dim=8,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2,
               loss_target=target, output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    rows = training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="eval", restart_backbone=True,
                                                   restart_head=True)).run()
    col = 1 if target == "energies" else 2
    assert all(np.isfinite(r[col]) for r in rows)
    assert (tmp_path / "model_energy_eval_0.txt").exists()


def test_state_dict_shapes_follow_reference_modules():
    """Every parameter/buffer shape of the backbone and Fock head equals the shape the
    reference's module definitions give (``esen_osh.py:140-200, 522-703``, ``esen_block.py:60-105,
    261-298``, ``so2_layers.py:19-214``, ``layer_norm.py:230-338``, e3nn ``o3.Linear`` flat
    weights), for the reference's own setting mmax = lmax and the source-target message."""
    _, lab = _batches(np.eye(3), torch.float32)
    L, C, Hd, Ce, G = 4, 8, 8, 8, 8
    kw = dict(KW, mmax=L)
    bb = eSEN_Backbone(lab.irreps, **kw)
    sd = {k: tuple(v.shape) for k, v in bb.state_dict().items()}
    Cin = 2 * C  # source-target message
    n_rad = (L + 1) * Cin + sum((L - m + 1) * Cin for m in range(1, L + 1))
    exp = {f"Jd_{l}": (2 * l + 1, 2 * l + 1) for l in range(L + 1)}
    exp.update({"distance_expansion.offset": (G,), "sphere_embedding.weight": (100, C),
                "charge_embedding.weight": (21, C), "spin_embedding.weight": (11, C),
                "scalar_node_embedding.weight": (C, 3 * C), "scalar_node_embedding.bias": (C,),
                "source_embedding.weight": (100, Ce), "target_embedding.weight": (100, Ce),
                "edge_degree_embedding.rad_func.net.0.weight": (Ce, G + 2 * Ce),
                "edge_degree_embedding.rad_func.net.1.weight": (Ce,),
                "edge_degree_embedding.rad_func.net.3.weight": (Ce, Ce),
                "edge_degree_embedding.rad_func.net.6.weight": ((L + 1) * C, Ce),
                "norm.affine_weight": (L + 1, C), "norm.affine_bias": (C,)})
    for kind in ("node_blocks", "edge_blocks"):
        for i in range(2):
            p = f"{kind}.{i}."
            exp.update({p + "norm_1.affine_weight": (L + 1, C), p + "norm_2.affine_bias": (C,),
                        p + "norm_1.balance_degree_weight": ((L + 1) ** 2, 1),
                        p + "edge_wise.so2_conv_1.fc_m0.weight": ((L + 1) * Hd + L * Hd, (L + 1) * Cin),
                        p + "edge_wise.so2_conv_1.fc_m0.bias": ((L + 1) * Hd + L * Hd,),
                        p + "edge_wise.so2_conv_1.rad_func.net.0.weight": (Ce, G + 2 * Ce),
                        p + "edge_wise.so2_conv_1.rad_func.net.6.weight": (n_rad, Ce),
                        p + "edge_wise.so2_conv_2.fc_m0.weight": ((L + 1) * C, (L + 1) * Hd),
                        p + "atom_wise.scalar_mlp.0.weight": (L * Hd, C),
                        p + "atom_wise.so3_linear_1.weight": (L + 1, Hd, C),
                        p + "atom_wise.so3_linear_2.weight": (L + 1, C, Hd),
                        p + "atom_wise.so3_linear_1.expand_index": ((L + 1) ** 2,)})
            for m in range(1, L + 1):
                exp[p + f"edge_wise.so2_conv_1.so2_m_conv.{m - 1}.fc.weight"] = (2 * Hd * (L - m + 1), (L - m + 1) * Cin)
                exp[p + f"edge_wise.so2_conv_2.so2_m_conv.{m - 1}.fc.weight"] = (2 * C * (L - m + 1), (L - m + 1) * Hd)
    for k, shape in exp.items():
        assert k in sd, k
        assert sd[k] == shape, (k, sd[k], shape)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=L, sphere_channels=C, ls_list=lab.layout.ls_list, reduce_node=True,
                          reduce_node_intra=True)
    hsd = {k: tuple(v.shape) for k, v in hd.state_dict().items()}
    # scalars C x 0e -> (C + L*C) x 0e (C scalars + one gate per gated irrep C x 1e .. C x Le)
    assert hsd["lin_scalars_learnable.0.weight"] == (C * (C + L * C),)  # e3nn flat [mul_in * mul_out]
    for l in range(L + 1):
        k = f"node_lin_out_layers.0.{l}.weight"
        if k in hsd:
            mul_out = hd.node_lin_out_layers[0][l].mul_out
            assert hsd[k] == (C * mul_out,), (k, hsd[k])


def test_loss_png_is_a_valid_image(tmp_path):
    import struct
    import zlib

    from maloq_b200.utils.lossplot import save_loss_png

    h = {"train_node": [1.0, 0.3, 0.05], "train_edge": [2.0, 0.5, 0.2], "val_node": [1.2, 0.4, 0.1],
         "val_edge": [float("nan"), 0.6, 0.3]}
    data = open(save_loss_png(str(tmp_path / "loss.png"), h), "rb").read()
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    w, hgt = struct.unpack(">II", data[16:24])
    n = struct.unpack(">I", data[33:37])[0]
    assert data[37:41] == b"IDAT"
    raw = zlib.decompress(data[41:41 + n])
    img = np.frombuffer(raw, dtype=np.uint8).reshape(hgt, w * 3 + 1)[:, 1:].reshape(hgt, w, 3)
    assert (img == np.array([31, 119, 180], dtype=np.uint8)).all(-1).sum() > 50  # the train_node curve


def test_workflow_infer_writes_every_batch(tmp_path):
    """train_or_eval='infer' on a molecule dataset writes a block-sparse Hamiltonian for every
    batch of the evaluation set; each matches the dense labels -> matrix conversion."""
    from maloq.train_utils import training_workflow
    from maloq_b200.data import datasets
    from maloq_b200.parallel.infer import load_partitioned_hamiltonian

    cfg = dict(dataset_name="synthetic_small", num_structures=10, num_train=6, num_val=4, batch_size=2,
               num_epochs=1, l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5,
               rcut_gaussian=5.0, mmax=2, output_folder=str(tmp_path), device="cpu", log_every=0)
    training_workflow.TrainingWorkflow(cfg).run()
    paths = training_workflow.TrainingWorkflow(dict(cfg, train_or_eval="infer", restart_backbone=True,
                                                    restart_head=True)).run()
    assert len(paths) == 2
    lab = datasets.labeler_for("small")
    for i in range(2):
        H = load_partitioned_hamiltonian(str(tmp_path / f"batch_{i:04d}"), lab).to_dense()
        assert H.shape[0] == H.shape[1] > 0 and np.allclose(H, H.T, atol=1e-5)


def test_standalone_muon_orthogonal_steps():
    """Muon alone: matrices only; a step moves along an orthogonalised direction (its singular
    values are all close to one, times the learning rate) and a least-squares fit improves."""
    import pytest

    from maloq_b200.train.loss import Muon

    with pytest.raises(ValueError):
        Muon([torch.nn.Parameter(torch.zeros(3))])
    torch.manual_seed(0)
    W = torch.nn.Parameter(torch.zeros(16, 32))
    A, T = torch.randn(64, 16), torch.randn(64, 32)
    opt = Muon([W], lr=0.05, momentum=0.0)
    loss0 = ((A @ W - T) ** 2).mean()
    loss0.backward()
    before = W.detach().clone()
    opt.step()
    sv = torch.linalg.svdvals((W.detach() - before) / 0.05)
    assert sv.min() > 0.5 and sv.max() < 1.5
    for _ in range(30):
        opt.zero_grad()
        ((A @ W - T) ** 2).mean().backward()
        opt.step()
    assert ((A @ W - T) ** 2).mean().item() < loss0.item()
