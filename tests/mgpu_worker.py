"""Multi-GPU test bodies, launched by the tests under torch.distributed.run (one process per GPU)."""

import sys

import torch
import torch.distributed as dist


def dp_nvlink() -> None:
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.engine.optim import AdamWConfig
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel.groups import init_distributed
    from tests.helpers import set_old_log_probs, tree_batch

    rank, world = init_distributed(timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = get_config("tiny", hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=1024,
                     num_layers=2)
    batch = tree_batch(n_trees=2, prefix=130, siblings=3, resp=70, seed=11 + rank)
    batch["dp_size"] = world
    opt = AdamWConfig(lr=1e-3, grad_clip=0.5)
    engines = {}
    for mode in ("nccl", "nvlink"):
        eng = TPREngine(cfg, EngineConfig(dp_comm=mode, grad_comm_dtype="fp32"), opt, device=dev,
                        model=build_model(cfg, device=dev, seed=0))
        set_old_log_probs(eng.model, batch)
        engines[mode] = eng
    total = torch.tensor([float(sum(int(m.sum()) for m in batch["response_mask"]))], device=dev)
    dist.all_reduce(total)
    batch["batch_num_tokens"] = int(total.item())
    init = {n: p.detach().float().clone() for n, p in engines["nccl"].model.named_parameters()}
    norms = {}
    for step in range(2):
        for mode, eng in engines.items():
            out = eng.train_step(batch)
            norms.setdefault(mode, []).append(float(out["grad_norm"]))
    assert engines["nvlink"].symm_heap is not None and engines["nccl"].symm_heap is None
    for a, b in zip(norms["nccl"], norms["nvlink"]):
        assert abs(a - b) <= 2e-2 * abs(a) + 1e-6, (norms)
    # Adam turns bf16 noise in near-zero gradients into +-lr steps, so compare the update directions
    pa = dict(engines["nccl"].model.named_parameters())
    da, db = [], []
    for n, p in engines["nvlink"].model.named_parameters():
        da.append((pa[n].float() - init[n]).flatten())
        db.append((p.float() - init[n]).flatten())
        # every rank ends with identical parameters
        g = [torch.empty_like(p) for _ in range(world)]
        dist.all_gather(g, p.detach().contiguous())
        assert all(torch.equal(g[0], x) for x in g[1:]), n
    da, db = torch.cat(da), torch.cat(db)
    cos = float(torch.nn.functional.cosine_similarity(da, db, dim=0))
    rel = float((da - db).norm() / da.norm())
    assert da.norm() > 0 and cos > 0.95 and rel < 0.3, (cos, rel)
    # the sharded optimizer state comes back in parameter order (the same layout as the replicated one)
    sa, sb = engines["nccl"].optimizer.state_dict(), engines["nvlink"].optimizer.state_dict()
    assert sa["step"] == sb["step"] == 2
    for x, y in zip(sa["arenas"], sb["arenas"]):
        assert x["master"].shape == y["master"].shape
        d = float((x["master"] - y["master"]).norm() / x["master"].norm())
        assert d < 1e-2, d
    # and loads back: a round trip leaves master / moments / parameters unchanged
    before = {n: p.detach().clone() for n, p in engines["nvlink"].model.named_parameters()}
    engines["nvlink"].optimizer.load_state_dict(sb)
    again = engines["nvlink"].optimizer.state_dict()
    for x, y in zip(sb["arenas"], again["arenas"]):
        for key in ("master", "m", "v"):
            assert torch.equal(x[key], y[key]), key
    for n, p in engines["nvlink"].model.named_parameters():
        assert torch.equal(p.detach(), before[n]), n
    engines["nvlink"].symm_heap.close()
    dist.barrier()
    if rank == 0:
        print("DP_NVLINK_OK", norms, cos, rel, flush=True)
    dist.destroy_process_group()


def tp_fused() -> None:
    """Fused all-gather+GEMM / GEMM+reduce-scatter linears vs the NCCL sequence-parallel path."""
    from bridge_b200.parallel.groups import init_distributed
    from bridge_b200.parallel.tp import gather_from_sp, reduce_scatter_to_sp
    from bridge_b200.ops.gemm import linear
    from bridge_b200.parallel import tp_fused as tf

    rank, world = init_distributed(timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    group = dist.group.WORLD
    tf.set_tp_comm_mode("nvlink")
    for ms, k, n_out in ((384, 512, 768), (200, 256, 520), (1152, 2560, 3072)):
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn(ms, k, device=dev, generator=g).bfloat16()
        w = (torch.randn(n_out, k, device=dev, generator=g) * 0.05).bfloat16()
        comm = tf.fused_comm(group, x)
        assert comm is not None
        # column-parallel: y = AG(x) W^T
        xa = x.clone().requires_grad_()
        wa = w.clone().requires_grad_()
        ya = tf.ag_linear(xa, wa, comm)
        xb = x.clone().requires_grad_()
        wb = w.clone().requires_grad_()
        yb = linear(gather_from_sp(xb, group), wb)
        dy = torch.randn(ya.shape, device=dev, generator=g).bfloat16()
        ya.backward(dy)
        yb.backward(dy)
        for name, a, b in (("y", ya, yb), ("dx", xa.grad, xb.grad), ("dw", wa.grad, wb.grad)):
            err = (a.float() - b.float()).abs().max().item()
            tol = 2e-2 * b.float().abs().max().item() + 1e-3
            assert err <= tol, ("ag", ms, name, err, tol)
        # row-parallel: y = RS(x_full W^T), x_full [ms*world, k]
        xf = torch.randn(ms * world, k, device=dev, generator=g).bfloat16()
        xa = xf.clone().requires_grad_()
        wa = w.clone().requires_grad_()
        ya = tf.linear_rs(xa, wa, comm)
        xb = xf.clone().requires_grad_()
        wb = w.clone().requires_grad_()
        yb = reduce_scatter_to_sp(linear(xb, wb), group)
        dy = torch.randn(ya.shape, device=dev, generator=g).bfloat16()
        ya.backward(dy)
        yb.backward(dy)
        for name, a, b in (("y", ya, yb), ("dx", xa.grad, xb.grad), ("dw", wa.grad, wb.grad)):
            err = (a.float() - b.float()).abs().max().item()
            tol = 2e-2 * b.float().abs().max().item() + 1e-3
            assert err <= tol, ("rs", ms, name, err, tol)
    torch.cuda.synchronize()
    from bridge_b200.ops._ext import kernels

    assert kernels().gemm_error_code() == 0 and kernels().symm_error_code() == 0
    tf.close_all()
    dist.barrier()
    if rank == 0:
        print("TP_FUSED_OK", flush=True)
    dist.destroy_process_group()


def cp_p2p() -> None:
    """TPR with CP over the NVLink P2P transport (ring zigzag and all-gather contiguous shards) vs the
    flattened batch on one GPU and vs the NCCL transport."""
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel import cp_p2p
    from bridge_b200.parallel.groups import build_parallel_state, init_distributed
    from tests.helpers import flat_ppo_loss, set_old_log_probs, tree_batch

    rank, world = init_distributed(timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = get_config("tiny", hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=1024,
                     num_layers=2)
    batch = tree_batch(n_trees=2, prefix=131, siblings=3, resp=77, seed=3)
    ref = build_model(cfg, device=dev, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    gref = {n: p.grad.float() for n, p in ref.named_parameters()}
    ps = build_parallel_state(tp=1, cp=world)
    results = {}
    import os

    combos = [(b, m) for b in ("ring", "allgather") for m in ("nvlink", "nccl")]
    if os.environ.get("CP_P2P_ONLY"):
        combos = [tuple(os.environ["CP_P2P_ONLY"].split(","))]
    for backend, mode in combos:
        if True:
            eng = TPREngine(cfg, EngineConfig(context_parallel_size=world, tpr_cp_backend=backend, cp_comm=mode,
                                              dp_comm="nccl"),
                            device=dev, model=build_model(cfg, device=dev, seed=0), parallel_state=ps)
            print(f"[r{rank}] start {backend} {mode}", file=sys.stderr, flush=True)
            out = eng.forward_backward_batch(batch)
            loss = float(out["loss"][0])
            print(f"[r{rank}] done {backend} {mode} loss={loss}", file=sys.stderr, flush=True)
            worst = 0.0
            for n, p in eng.model.named_parameters():
                a = p.main_grad.float()
                rel = float((a - gref[n]).norm() / (gref[n].norm() + 1e-12))
                worst = max(worst, rel)
            results[(backend, mode)] = (loss, worst)
            assert abs(loss - float(loss_ref)) <= 5e-3 * abs(float(loss_ref)) + 1e-4, (backend, mode, loss,
                                                                                        float(loss_ref))
            assert worst < 5e-2, (backend, mode, worst)
    if any(m == "nvlink" for _, m in combos):
        assert cp_p2p._COMMS, "the P2P transport was not used"
    cp_p2p.close_all()
    dist.barrier()
    if rank == 0:
        print("CP_P2P_OK", results, float(loss_ref), flush=True)
    dist.destroy_process_group()


def ep_p2p() -> None:
    """MoE layer with EP over the NVLink P2P dispatch/combine vs the NCCL all-to-all path and vs the
    unsharded layer (all experts on every rank)."""
    from bridge_b200.models import get_config
    from bridge_b200.models.moe import MoELayer
    from bridge_b200.parallel import ep_p2p
    from bridge_b200.parallel.groups import init_distributed

    rank, world = init_distributed(timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    group = dist.group.WORLD
    cfg = get_config("tiny_moe", hidden_size=256, moe_intermediate_size=128, num_experts=8, moe_top_k=3)
    torch.manual_seed(0)
    full = MoELayer(cfg, device=dev)
    with torch.no_grad():
        full.router.mul_(20.0)
    el = cfg.num_experts // world
    x = torch.randn(257 + 31 * rank, 256, device=dev, generator=torch.Generator(device=dev).manual_seed(rank)).bfloat16()
    dy = torch.randn(x.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(50 + rank)).bfloat16()
    xf = x.clone().requires_grad_()
    yf = full(xf)
    yf.backward(dy)
    gfull = {n: p.grad.float() for n, p in full.named_parameters()}
    for n in ("w1", "w2"):
        dist.all_reduce(gfull[n], group=group)          # expert grads see every rank's tokens under EP
    for mode in ("nvlink", "nccl"):
        ep_p2p.set_ep_comm_mode(mode)
        torch.manual_seed(0)
        layer = MoELayer(cfg, ep_group=group, device=dev)
        with torch.no_grad():
            layer.router.copy_(full.router)
            layer.w1.copy_(full.w1[rank * el:(rank + 1) * el])
            layer.w2.copy_(full.w2[rank * el:(rank + 1) * el])
            for n in ("shared_w1", "shared_w2", "shared_gate"):
                getattr(layer, n).copy_(getattr(full, n))
        xe = x.clone().requires_grad_()
        ye = layer(xe)
        ye.backward(dy)
        def close(a, b, name):
            err = (a.float() - b.float()).abs().max().item()
            tol = 2e-2 * b.float().abs().max().item() + 1e-3
            assert err <= tol, (mode, name, err, tol)
        close(ye, yf, "y")
        close(xe.grad, xf.grad, "dx")
        close(layer.w1.grad, gfull["w1"][rank * el:(rank + 1) * el], "dw1")
        close(layer.w2.grad, gfull["w2"][rank * el:(rank + 1) * el], "dw2")
    assert ep_p2p._COMMS, "P2P dispatch was not used"
    ep_p2p.close_all()
    dist.barrier()
    if rank == 0:
        print("EP_P2P_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    import os

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    {"dp_nvlink": dp_nvlink, "tp_fused": tp_fused, "cp_p2p": cp_p2p, "ep_p2p": ep_p2p}[sys.argv[1]]()
