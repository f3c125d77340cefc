"""Fused peer-memory reduce-scatter on 2 GPUs (NCCL ranks): the kernel against
NCCL's reduce_scatter, and FSDP training with fused gradients against the same
run on NCCL's reduce-scatter."""
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from rl_project_b200.parallel.runtime import free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multi_gpu]
# every GPU of the box (2 to 8); one rank per GPU
WORLD = max(2, min(8, torch.cuda.device_count())) if torch.cuda.is_available() else 2
STEPS = 3
MODES = ("off", "on")  # CUDA IPC mappings + peer loads; symmetric memory + NVLink multicast reduce


def _env(rank, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank))


def _kernel_worker(rank, port, out):
    import datetime

    import torch.distributed as dist

    from rl_project_b200.parallel.fused_comm import FusedReduceScatter

    _env(rank, port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    res = {}
    for mc in MODES:
        shard = 1 << 18
        fr = FusedReduceScatter(None, shard * WORLD, torch.device("cuda", rank), multicast=mc, timeout_s=20.0)
        errs = []
        for it in range(6):  # more uses than slots: exercises the ring and its reuse rule
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            x = torch.randn(WORLD * shard, device="cuda", generator=g).bfloat16()
            slot = fr.next_slot(WORLD * shard)
            slot.copy_(x)
            outp = torch.empty(shard, device="cuda")
            fr.reduce(shard, outp, False, True)
            ref = torch.empty(shard, dtype=torch.float32, device="cuda")
            dist.reduce_scatter_tensor(ref, x.float())
            ref /= WORLD
            # the multicast reduce returns bf16 sums (fp32 accumulation): allow one bf16 ulp of the result
            tol = 1e-5 if mc == "off" else 2.0 ** -7 * max(1.0, float(ref.abs().max()))
            errs.append(float((outp - ref).abs().max()) / tol)
        torch.cuda.synchronize()
        fr.poll_status()
        torch.cuda.synchronize()
        fr.check()
        res[mc] = {"err": max(errs), "multicast": fr.uses_multicast}
        fr.close()
        del fr
    torch.save(res, os.path.join(out, f"k{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_fused_kernel_matches_nccl():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_kernel_worker, args=(free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
        for r in range(WORLD):
            res = torch.load(os.path.join(out, f"k{r}.pt"))
            for mc, v in res.items():
                assert v["err"] <= 1.0, (r, mc, v)


def _train_worker(rank, port, out, mode):
    from rl_project_b200.core.config import ExperimentManifest
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel.strategies import build_strategy
    from rl_project_b200.training.common.trainer import Trainer
    from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig

    _env(rank, port)
    torch.cuda.set_device(rank)
    m = ExperimentManifest.from_dict({
        "name": "t", "algorithm": "pretrain", "model_preset": "tiny", "model": {"vocab_size": 4096, "block_size": 64},
        "trainer": {"device": f"cuda:{rank}", "precision": {"dtype": "bfloat16"}, "eval_every": 0, "log_every": 0,
                    "max_steps": STEPS, "batch_size": 4, "gradient_accumulation_steps": 2,
                    "optimizer": {"learning_rate": 1e-3, "grad_clip": 0.5},
                    "schedule": {"name": "constant", "warmup_steps": 0}, "checkpoint": {"save_every": 0}},
        "distributed": {"strategy": "fsdp", "backend": "nccl", "timeout_s": 60, "fused_comm": mode},
        "output_dir": os.path.join(out, f"{mode}{rank}")})
    strat = build_strategy(m.distributed)
    strat.setup()
    ctx = RunContext.create(m, metrics_backend="none", distributed=False, device_override=f"cuda:{rank}")
    torch.manual_seed(0)
    model = TransformerLM(m.model).to(ctx.device)
    g = torch.Generator().manual_seed(11 + rank)

    class It:
        def __iter__(self):
            return self

        def __next__(self):
            b = torch.randint(0, 4096, (4, 65), generator=g)
            return b[:, :-1].to(ctx.device), b[:, 1:].to(ctx.device)

    alg = PretrainAlgorithm(model, It(), PretrainConfig(batch_size=4), device=ctx.device)
    trainer = Trainer(ctx, alg, strategy=strat)
    res = [trainer.train_step() for _ in range(STEPS)]
    fused = strat.fused is not None
    state = strat.full_state_dict()
    torch.save({"losses": [r.loss for r in res], "norms": [r.metrics["grad_norm"] for r in res], "state": state,
                "fused": fused}, os.path.join(out, f"{mode}{rank}.pt"))
    strat.teardown()


def test_fsdp_fused_gradients_match_nccl():
    with tempfile.TemporaryDirectory() as out:
        for mode in ("on", "nccl_baseline"):
            mp.start_processes(_train_worker, args=(free_port(), out, mode), nprocs=WORLD, join=True,
                               start_method="spawn")
        a = torch.load(os.path.join(out, "on0.pt"))
        b = torch.load(os.path.join(out, "nccl_baseline0.pt"))
    assert a["fused"] and not b["fused"]
    for x, y in zip(a["losses"], b["losses"]):
        assert abs(x - y) < 2e-2 * max(1.0, abs(y))
    for x, y in zip(a["norms"], b["norms"]):
        assert abs(x - y) < 2e-2 * max(1.0, abs(y))
    for k, v in b["state"].items():
        d = (a["state"][k] - v).abs().max().item()
        assert d < 5e-3, (k, d)


def _bcast_worker(rank, port, out):
    import datetime

    import torch.distributed as dist

    from rl_project_b200.parallel.weight_sync import ParameterBroadcaster

    _env(rank, port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    res = {}
    for mc in ("on", "off"):
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        ts = [torch.randn(1000003, device="cuda", generator=g).bfloat16(),
              torch.randn(257, 129, device="cuda", generator=g),
              torch.randint(0, 1 << 30, (4097,), device="cuda", generator=g)]
        b = ParameterBroadcaster(None, device=torch.device("cuda", rank), chunk_bytes=1 << 20, multicast=mc)
        b.broadcast_(ts, src=1)
        torch.cuda.synchronize()
        res[mc] = {"mode": b.mode, "sums": [float(t.double().sum()) for t in ts],
                   "first": [t.reshape(-1)[:4].double().tolist() for t in ts]}
        del b
    torch.save(res, os.path.join(out, f"b{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_parameter_broadcast_nvls_and_nccl():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_bcast_worker, args=(free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
        r0, r1 = torch.load(os.path.join(out, "b0.pt")), torch.load(os.path.join(out, "b1.pt"))
    assert r0["on"]["mode"] == "nvls" and r0["off"]["mode"] == "nccl"
    for mc in ("on", "off"):
        assert r0[mc]["sums"] == r1[mc]["sums"] and r0[mc]["first"] == r1[mc]["first"], mc


def _tp_worker(rank, port, out):
    import datetime

    import torch.distributed as dist

    from rl_project_b200.parallel.tp_fused import GemmAllReduce

    _env(rank, port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    red = GemmAllReduce(None, 4096 * 1024, torch.device("cuda", rank))
    res = []
    for it, (M, N, K) in enumerate([(1000, 512, 256), (4096, 1024, 384), (130, 288, 64), (4096, 1024, 384),
                                    (1000, 512, 256)]):  # more launches than slots, mixed shapes
        g = torch.Generator(device="cuda").manual_seed(1000 * it + rank)
        x = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
        w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
        dy = (torch.randn(M, N, device="cuda", generator=g) / N ** 0.5).bfloat16()
        y = red(x, w)  # row-parallel output: sum_r x_r @ w_r^T
        dx = red.dgrad(dy, w)  # column-parallel input gradient: sum_r dy_r @ w_r (B stored [K][N])
        for out_, part in ((y, x.float() @ w.float().t()), (dx, dy.float() @ w.float())):
            ref = part.bfloat16().float()  # each rank's partial, rounded like the kernel's
            dist.all_reduce(ref)
            err = float((out_.float() - ref).abs().max() / ref.abs().max())
            digest = torch.tensor([float(out_.float().double().sum())], device="cuda", dtype=torch.float64)
            all_d = [torch.zeros_like(digest) for _ in range(WORLD)]
            dist.all_gather(all_d, digest)
            res.append({"err": err, "identical": len({float(d) for d in all_d}) == 1, "shape": (M, N, K)})
    torch.cuda.synchronize()
    red.check()
    red.close()
    torch.save(res, os.path.join(out, f"tp{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_gemm_allreduce_matches_nccl():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_tp_worker, args=(free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
        res = torch.load(os.path.join(out, "tp0.pt"))
    for r in res:
        assert r["identical"], res
        assert r["err"] < 2e-2, res  # bf16 partials: the kernel's and cuBLAS's roundings may differ by an ulp


def _tp_model_worker(rank, port, out):
    """Tensor parallelism over every rank: fused epilogue all-reduces (row-parallel forward and
    column-parallel input gradients) against NCCL all-reduces, same weights and batch."""
    import datetime

    import torch.distributed as dist

    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.transformer.model import TransformerLM
    from rl_project_b200.parallel import tp_fused
    from rl_project_b200.parallel.tensor_parallel import apply_tensor_parallel

    _env(rank, port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    spec = model_spec_from_preset("bl_tiny", n_layer=2, n_head=8, n_kv_head=8, n_embd=512, d_ff=1024,
                                  block_size=256, vocab_size=1024, dropout=0.0)
    torch.manual_seed(0)
    base = TransformerLM(spec)
    x = torch.randint(0, spec.vocab_size, (2, 256), generator=torch.Generator().manual_seed(5)).cuda()
    y = torch.roll(x, -1, 1)
    runs = {}
    for fused in (False, True):
        tp_fused.set_enabled(fused)
        m = TransformerLM(spec)
        m.load_state_dict(base.state_dict())
        m = apply_tensor_parallel(m, dist.group.WORLD, rank, WORLD).cuda().to(torch.bfloat16)
        _, loss = m(x, y)
        loss.backward()
        runs[fused] = (float(loss), {n: p.grad.float().clone() for n, p in m.named_parameters()})
        torch.cuda.synchronize()
    red = tp_fused._REDUCERS.get(dist.group.WORLD)
    used = red is not None and red.launches > 0
    if red is not None:
        red.check()
    tp_fused.close_all()
    tp_fused.set_enabled(True)
    worst = 0.0
    for n, g0 in runs[False][1].items():
        g1 = runs[True][1][n]
        worst = max(worst, float((g1 - g0).norm() / g0.norm().clamp(min=1e-12)))
    torch.save({"loss": (runs[False][0], runs[True][0]), "grad_rel": worst, "used": used,
                "launches": red.launches if red is not None else 0}, os.path.join(out, f"tpm{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_tensor_parallel_model_fused_matches_nccl():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_tp_model_worker, args=(free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
        res = [torch.load(os.path.join(out, f"tpm{r}.pt")) for r in range(WORLD)]
    for r in res:
        assert r["used"], res
        # 2 layers x (q|k|v dgrad, w1|w3 dgrad, attention-out and w2 forward) fused launches per step
        assert r["launches"] == 2 * 4, res
        a, b = r["loss"]
        assert abs(a - b) < 1e-2 * abs(a), res
        assert r["grad_rel"] < 3e-2, res


def _ep_worker(rank, port, out):
    import datetime

    import torch.distributed as dist

    from rl_project_b200.core.config import model_spec_from_preset
    from rl_project_b200.models.moe.layer import MoELayer
    from rl_project_b200.parallel import expert_p2p
    from rl_project_b200.parallel.expert import shard_experts

    _env(rank, port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    torch.manual_seed(0)
    spec = model_spec_from_preset("tiny", vocab_size=97, use_moe=True, n_experts=8, n_experts_active=2,
                                  n_embd=128, moe_d_ff=192, n_shared_experts=1)
    layer = MoELayer(spec).cuda().bfloat16()
    shard_experts(layer, dist.group.WORLD, rank, WORLD)
    g = torch.Generator(device="cuda").manual_seed(rank)
    x = torch.randn(2, 96, 128, device="cuda", generator=g).bfloat16()
    dy = torch.randn(2, 96, 128, device="cuda", generator=g).bfloat16()
    res = {}
    for mode in (True, False, True):
        expert_p2p.set_enabled(mode)
        layer.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(True)
        y = layer(xi)
        y.backward(dy)
        res.setdefault(mode, []).append((y.float(), xi.grad.float(),
                                         {n: p.grad.float().clone() for n, p in layer.named_parameters()
                                          if p.grad is not None}))
    torch.cuda.synchronize()
    used = bool(expert_p2p._RINGS)
    for r in expert_p2p._RINGS.values():
        r.check()
    expert_p2p.close_all()
    (yp, dxp, gp), (yn, dxn, gn) = res[True][0], res[False][0]
    errs = {"y": float((yp - yn).abs().max()), "dx": float((dxp - dxn).abs().max()),
            "params": max(float((gp[n] - gn[n]).abs().max() / (gn[n].abs().max() + 1e-6)) for n in gn),
            "same_params": set(gp) == set(gn), "used": used,
            "repeat": float((res[True][1][0] - yp).abs().max())}
    torch.save(errs, os.path.join(out, f"ep{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_p2p_matches_nccl():
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_ep_worker, args=(free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
        errs = [torch.load(os.path.join(out, f"ep{r}.pt")) for r in range(WORLD)]
    for e in errs:
        assert e["used"] and e["same_params"], e
        assert e["y"] < 1e-2 and e["dx"] < 1e-2 and e["repeat"] == 0.0, e
        assert e["params"] < 2e-2, e
