"""Data-parallel paths.

CPU (gloo, 2 ranks): the reference semantics of averaging gradients after
backward, host-side shard tables.  GPU (1 device): the fused kernels' bounded
waits time out into an error status instead of hanging when a peer never
arrives (the "peer" flag is a local buffer nothing writes).  Multi-GPU
(2 devices): the fused NVSwitch step matches the NCCL baseline.
"""
import math
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mmltk_b200.parallel.fused import shard_chunks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_chunks_cover_each_element_once():
    chunks = torch.tensor([[0, 128, 0], [128, 64, 1], [192, 256, 0], [448, 64, 2]])
    total, world = 512, 4
    S = total // world
    seen = torch.zeros(total, dtype=torch.int32)
    for r in range(world):
        t = shard_chunks(chunks, r * S, S)
        for o, n, g in t.tolist():
            seen[r * S + o:r * S + o + n] += 1
            # group of every element is preserved
            for e in range(r * S + o, r * S + o + n):
                gg = [c[2] for c in chunks.tolist() if c[0] <= e < c[0] + c[1]]
                assert gg == [g]
    assert (seen == 1).all()


def _cpu_ddp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from mmltk_b200.config import TrainOptions, config_from_preset
    from mmltk_b200.data.synthetic import synthetic_batch
    from mmltk_b200.models import RFDETR
    from mmltk_b200.parallel.ddp import NcclGradSync
    from mmltk_b200.train.engine import TrainEngine
    torch.manual_seed(0)
    model = RFDETR(config_from_preset("rf-detr-tiny-test", resolution=64))
    eng = TrainEngine(model, TrainOptions(lr=1e-3), "cpu", grad_sync=NcclGradSync(), max_targets=4)
    imgs, tg = synthetic_batch(2, 64, seed=100 + rank, kmax=4, slots=4)  # different data per rank
    for _ in range(2):
        eng.step(imgs, tg)
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    out = [torch.zeros_like(flat) for _ in range(world)]
    dist.all_gather(out, flat)
    q.put((rank, float((out[0] - out[1]).abs().max())))
    dist.destroy_process_group()


def test_bucket_plan_and_rank_slices_cover_each_element_once():
    """Buckets of a backward-ordered flat buffer tile it exactly, fire from its end, and every
    rank's 64-aligned slices of them tile each bucket exactly (any world size)."""
    from mmltk_b200.parallel.fused import plan_buckets, rank_slices
    total = 1000 * 64
    bounds = [640 + 64 * 50 * i for i in range(12)]           # mark i completes [bounds[i], total)
    buckets = plan_buckets(total, bounds, 64 * 120)
    assert buckets[0][2] == total and buckets[-1][0] is None and buckets[-1][1] == 0
    for (m0, a0, b0), (m1, a1, b1) in zip(buckets, buckets[1:]):
        assert a0 == b1                                          # contiguous, firing towards the start
        assert m1 is None or m1 < m0
    for world in (1, 2, 3, 8):
        cover = sorted(x for r in range(world) for x in rank_slices(buckets, world, r))
        pos = 0
        for a, b in cover:
            assert a == pos and a % 64 == 0
            pos = b
        assert pos == total


def test_flat_layout_follows_backward_stages():
    """With a stage function the flat buffer holds later-completing (earlier) stages first, so the
    gradients one ViT layer completes are contiguous."""
    from mmltk_b200.config import config_from_preset
    from mmltk_b200.models import RFDETR
    from mmltk_b200.train.flat import FlatParams
    m = RFDETR(config_from_preset("rf-detr-nano"))
    named = [(n, p) for n, p in m.named_parameters()]
    flat = FlatParams(named, [0] * len(named), "cpu", torch.float32, stage=m.grad_stage)
    stages = [m.grad_stage(n) for n in flat.names]
    assert stages == sorted(stages)
    assert flat.offsets == sorted(flat.offsets)
    assert m.grad_mark_count() == len(m.backbone[0].encoder.encoder.encoder.layer)


def test_cpu_gloo_ddp_keeps_ranks_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(d == 0.0 for _, d in res)


@pytest.mark.gpu
def test_fused_wait_times_out_into_status(cuda_device):
    """A peer that never signals: the kernel gives up after spin_limit polls and reports it."""
    from mmltk_b200.ops import kernels
    k = kernels()
    n = 4096
    own = [k.ipc_alloc(n * 2, 0)[0] for _ in range(2)]          # param, grad
    fake = [k.ipc_alloc(n * 2, 0)[0] for _ in range(2)]          # the "peer's" buffers (local, never signalled)
    flags, _ = k.ipc_alloc(k.ddp_flag_words() * 4, 0)
    fake_flags, _ = k.ipc_alloc(k.ddp_flag_words() * 4, 0)
    small, _ = k.ipc_alloc(k.ddp_small_floats() * 4, 0)
    fake_small, _ = k.ipc_alloc(k.ddp_small_floats() * 4, 0)
    ctrl = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    ctrl[0] = 1
    ctrl[1] = 1
    comm = k.DdpComm([own[1].data_ptr(), fake[1].data_ptr()], [own[0].data_ptr(), fake[0].data_ptr()],
                     [flags.data_ptr(), fake_flags.data_ptr()], [small.data_ptr(), fake_small.data_ptr()],
                     0, 2, flags.view(torch.int32), small.view(torch.float32), ctrl, 2000)
    gshard = torch.zeros(n // 2, device=cuda_device)
    blocks = k.ddp_rs_blocks(True)
    partials = torch.zeros(blocks, device=cuda_device)
    comm.rs(0, n // 2, gshard, 0, partials, 0, 0, blocks)       # bucket 0 of step epoch 1
    torch.cuda.synchronize()
    assert int(ctrl[3]) == 1  # timed out waiting for 'bucket ready'
    # our own 'bucket ready' mark (epoch * 32 + bucket + 1) was delivered to the fake peer
    assert int(fake_flags.view(torch.int32)[0]) == 33
    ctrl[3] = 0
    data = torch.ones(3, device=cuda_device)
    comm.small_allreduce(data)
    torch.cuda.synchronize()
    assert int(ctrl[3]) == 4
    ctrl[3] = 0
    ctrl[4] = 1
    out = torch.zeros(64, dtype=torch.uint8, device=cuda_device)
    comm.gather_bytes(out, [0, 1], [1, 1])
    torch.cuda.synchronize()
    assert int(ctrl[3]) == 5  # the peer never staged its payload for the byte all-gather


def _oracle_update(master, m, v, ema, grad_sum, elem_lr, elem_wd, sc):
    """fp32 statement of one optimizer step on the summed gradient: average, global-norm clip,
    AdamW (decoupled weight decay), EMA -- the semantics both gradient paths must implement
    (reference `train.cpp:2295-2344`, `native_optimizer.cpp:401-410`, `training_ops.h:186-204`)."""
    lr_scale, b1, b2, eps, bc1, bc2, max_norm, ema_d, ema_on, inv_world = sc[:10].tolist()
    g = grad_sum * inv_world
    norm = g.norm()
    if max_norm > 0:
        g = g * torch.clamp(max_norm / (norm + 1e-6), max=1.0)
    m2 = b1 * m + (1 - b1) * g
    v2 = b2 * v + (1 - b2) * g * g
    lr = elem_lr * lr_scale
    master2 = master * (1 - lr * elem_wd) - lr / bc1 * m2 / (v2.sqrt() / math.sqrt(bc2) + eps)
    ema2 = ema_d * ema + (1 - ema_d) * master2 if ema_on else ema
    return master2, m2, v2, ema2


def _gpu_ddp_worker(rank, world, port, backend, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    from mmltk_b200.config import TrainOptions, config_from_preset
    from mmltk_b200.data.synthetic import synthetic_batch
    from mmltk_b200.models import RFDETR
    from mmltk_b200.parallel.ddp import NcclGradSync
    from mmltk_b200.parallel.fused import FusedGradSync
    from mmltk_b200.train.engine import TrainEngine
    torch.manual_seed(0)
    cfg = config_from_preset("rf-detr-medium", group_detr=2, dec_layers=2, resolution=256,
                             positional_encoding_size=16)
    sync = FusedGradSync() if backend == "fused" else NcclGradSync()
    eng = TrainEngine(RFDETR(cfg), TrainOptions(lr=1e-3, lr_encoder=1.5e-3, use_ema=True, cuda_graph=True), "cuda",
                      grad_sync=sync, max_targets=6)
    eng.bind_static_inputs(2, 3, 256, 256)
    imgs, tg = synthetic_batch(2, 256, seed=10 + rank, kmax=6, slots=6, dtype=torch.bfloat16)
    imgs, tg = imgs.cuda(), tg.to("cuda")
    fused = backend == "fused"

    def full(t):       # optimizer state as full flat fp32 vectors
        return sync.gather_full(t) if fused else t.clone()

    def state():
        return [full(eng.master_shard if fused else eng.master), full(eng.m), full(eng.v), full(eng.ema_buf)]

    # element-wise lr / weight decay of the flat layout
    P = eng.flat.param_buf.numel()
    elem_lr = torch.zeros(P, device="cuda")
    elem_wd = torch.zeros(P, device="cuda")
    for o, n, g in eng.flat.chunk_table().tolist():
        elem_lr[o:o + n] = eng.group_hyper[g, 0]
        elem_wd[o:o + n] = eng.group_hyper[g, 1]

    report = []
    for step in range(4):            # steps 0-2 run eagerly, step 3 is the captured graph's first replay
        before = state()
        loss = eng.step(imgs, tg).loss
        after = state()
        if fused:
            # the kernel reads every rank's local bf16 gradient and accumulates in fp32
            grads = [torch.zeros_like(eng.flat.grad_buf) for _ in range(world)]
            dist.all_gather(grads, eng.flat.grad_buf)
            gsum = sum(g.float() for g in grads)
        else:
            gsum = eng.flat.grad_buf.float()     # NCCL summed in place, in the bf16 buffer
        sc = eng.scalars.float().cpu()
        om, omm, ov, oema = _oracle_update(*before, gsum, elem_lr, elem_wd, sc)
        upd = (om - before[0]).abs().max().item()
        rel = lambda a, b: ((a - b).abs() / (b.abs() + 1e-6)).max().item()
        # the master's error against the size of the numbers the update combined (a master value that
        # the update nearly cancels is accurate to the ulp of its inputs, not of the small result)
        mrel = lambda a, b, b0: ((a - b).abs() / (b.abs() + b0.abs() + 1e-6)).max().item()
        pb = eng.flat.param_buf
        # the bf16 parameters are the master rounded: within one bf16 ulp (2^-8 relative) at the scale
        # of the numbers the update combined
        ulps = ((pb.float() - om).abs() / (om.abs() + before[0].abs() + 1e-6)).max().item() * 256.0
        others = [torch.zeros_like(pb) for _ in range(world)]
        dist.all_gather(others, pb)
        same = all(torch.equal(others[0], o) for o in others[1:])
        report.append(dict(step=step, loss=loss, update=upd, master_err=((after[0] - om).abs()).max().item(),
                           master_rel=mrel(after[0], om, before[0]), m_rel=mrel(after[1], omm, before[1]),
                           v_rel=rel(after[2], ov),
                           ema_err=(after[3] - oema).abs().max().item(), param_ulps=ulps, ranks_equal=same))
    if fused:
        # evaluation-style byte all-gather over the gradient buffers (between steps), then one more
        # step that must still match the oracle (the step clears the staged bytes first)
        mine = torch.arange((rank + 3) * 5, dtype=torch.float64).view(-1, 5) + 1000 * rank
        parts = sync.all_gather_tensor(mine)
        gathered_ok = len(parts) == world and all(
            torch.equal(parts[j], torch.arange((j + 3) * 5, dtype=torch.float64).view(-1, 5) + 1000 * j)
            for j in range(world))
        empty_ok = all(p.shape == (0, 5) for p in sync.all_gather_tensor(torch.zeros(0, 5, dtype=torch.float64)))
        # the in-kernel gradient all-reduce (Muon's sync): every rank's buffer ends as the bf16 rounding
        # of the fp32 sum in rank order, bit for bit
        gen = torch.Generator(device="cuda").manual_seed(100 + rank)
        mine_g = torch.randn(eng.flat.grad_buf.numel(), device="cuda", generator=gen).bfloat16()
        every = [torch.zeros_like(mine_g) for _ in range(world)]
        dist.all_gather(every, mine_g)
        eng.flat.grad_buf.copy_(mine_g)
        sync.all_reduce_grads(eng)
        torch.cuda.synchronize()
        expect = every[0].float()
        for t in every[1:]:
            expect = expect + t.float()
        allreduce_ok = torch.equal(eng.flat.grad_buf, expect.bfloat16()) and int(sync.ctrl[3]) == 0
        gathered_ok = gathered_ok and allreduce_ok
        before = state()
        loss = eng.step(imgs, tg).loss
        after = state()
        grads = [torch.zeros_like(eng.flat.grad_buf) for _ in range(world)]
        dist.all_gather(grads, eng.flat.grad_buf)
        om, _, _, _ = _oracle_update(*before, sum(g.float() for g in grads), elem_lr, elem_wd,
                                     eng.scalars.float().cpu())
        report.append(dict(step=4, loss=loss, update=(om - before[0]).abs().max().item(),
                           master_err=((after[0] - om).abs()).max().item(),
                           master_rel=((after[0] - om).abs() / (om.abs() + before[0].abs() + 1e-6)).max().item(),
                           m_rel=0.0,
                           v_rel=0.0, ema_err=0.0, param_ulps=0, ranks_equal=gathered_ok and empty_ok))
    q.put((rank, report))
    eng.release_graph()
    if fused:
        sync.close()
    dist.barrier()
    dist.destroy_process_group()


def _run_gpu_ddp(backend):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_ddp_worker, args=(r, 2, port, backend, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("backend", ["fused", "nccl"])
def test_ddp_step_matches_fp32_oracle(backend):
    """Each step of either gradient path equals an fp32 oracle applied to the all-gathered bf16
    gradients and the state before the step (eager steps and a CUDA-graph replay): master / Adam
    moments / EMA to 1e-5 relative, bf16 parameters to 1 ulp of the oracle's master (both at the scale
    of the update's inputs, so that a value the update nearly cancels is not held to the ulp of the
    small result), every rank
    identical.  The update itself is ~1e-3, so a step that changed nothing would fail."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_gpu_ddp(backend)
    for rank, report in res:
        for r in report:
            assert math.isfinite(r["loss"]), r
            assert r["update"] > 1e-4, r
            # 3e-5: a master value near zero whose gradient is near zero takes an Adam step in the
            # epsilon regime, where the kernel's flushed denormals and the CPU oracle's kept ones differ
            assert r["master_rel"] < 3e-5 and r["master_err"] < 1e-3 * r["update"], r
            assert r["m_rel"] < 1e-4 and r["v_rel"] < 1e-4, r
            assert r["ema_err"] < 1e-5, r
            assert r["param_ulps"] <= 1.0, r
            assert r["ranks_equal"], r


def test_launcher_fails_fast_when_a_rank_dies(tmp_path):
    """Host-side failure injection: rank 1 exits with an error before the first collective; the
    launcher returns its code and terminates rank 0, which is blocked in a gloo barrier."""
    import sys
    import time
    from mmltk_b200.parallel.launch import launch_workers
    script = tmp_path / "worker.py"
    script.write_text(
        "import sys, datetime, torch.distributed as dist\n"
        "a = sys.argv\n"
        "rank = int(a[a.index('--dist-rank') + 1]); world = int(a[a.index('--dist-world-size') + 1])\n"
        "store = a[a.index('--dist-store-file') + 1]\n"
        "if rank == 1:\n"
        "    sys.exit(3)\n"
        "dist.init_process_group('gloo', store=dist.FileStore(store, world), rank=rank, world_size=world,\n"
        "                        timeout=datetime.timedelta(seconds=120))\n"
        "dist.barrier()\n")
    t0 = time.time()
    code = launch_workers(["--workers", "2"], [0, 1], entry=[sys.executable, str(script)])
    assert code == 3
    assert time.time() - t0 < 60


def test_worker_argv_rewrite():
    from mmltk_b200.parallel.launch import rewrite_worker_argv
    argv = ["rfdetr", "train", "--device-ids", "0,1", "--workers", "8", "--epochs", "2", "--dist-worker"]
    out = rewrite_worker_argv(argv, 1, 2, 1, "/tmp/s", 4)
    assert out[:4] == ["rfdetr", "train", "--epochs", "2"]
    assert out[out.index("--dist-rank") + 1] == "1" and out[out.index("--device-id") + 1] == "1"
    assert out.count("--workers") == 1 and out[out.index("--workers") + 1] == "4"


def _muon_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, ROOT)
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    from mmltk_b200.config import TrainOptions, config_from_preset
    from mmltk_b200.data.synthetic import synthetic_batch
    from mmltk_b200.models import RFDETR
    from mmltk_b200.parallel.fused import FusedGradSync
    from mmltk_b200.train.engine import TrainEngine
    torch.manual_seed(0)
    cfg = config_from_preset("rf-detr-medium", group_detr=2, dec_layers=2, resolution=256,
                             positional_encoding_size=16)
    sync = FusedGradSync()
    eng = TrainEngine(RFDETR(cfg), TrainOptions(optimizer="muon", lr=1e-3, use_ema=True, cuda_graph=False), "cuda",
                      grad_sync=sync, max_targets=6)
    eng.bind_static_inputs(2, 3, 256, 256)
    imgs, tg = synthetic_batch(2, 256, seed=20 + rank, kmax=6, slots=6, dtype=torch.bfloat16)
    before = eng.flat.param_buf.clone()
    losses = [eng.step(imgs.cuda(), tg.to("cuda")).loss for _ in range(3)]
    pb = eng.flat.param_buf
    others = [torch.zeros_like(pb) for _ in range(world)]
    dist.all_gather(others, pb)
    q.put((rank, dict(losses=losses, moved=(pb.float() - before.float()).abs().max().item(),
                      same=all(torch.equal(others[0], o) for o in others[1:]), status=int(sync.ctrl[3]))))
    sync.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_muon_with_fused_sync_keeps_ranks_identical():
    """Muon (replicated master weights) with the in-kernel gradient all-reduce: three steps, every
    rank's parameters identical and updated, finite losses, no wait gave up."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_muon_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, r in res:
        assert all(math.isfinite(x) for x in r["losses"]), r
        assert r["moved"] > 1e-5 and r["same"] and r["status"] == 0, r
