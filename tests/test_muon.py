"""Muon with auxiliary AdamW: orthogonalisation, eligibility, per-parameter
semantics (incl. the fused q/k/v weight as three matrices), loop + resume."""
import json
import math

import pytest
import torch

from mmltk_b200.train.muon import MuonAux, is_muon_hidden_weight, newton_schulz5


def test_newton_schulz_orthogonalises():
    torch.manual_seed(0)
    g = torch.randn(3, 64, 32)
    o = newton_schulz5(g).float()
    s = torch.linalg.svdvals(o)
    assert s.min() > 0.5 and s.max() < 1.3        # the quintic maps every singular value near 1
    o1 = newton_schulz5(g[1]).float()
    assert torch.allclose(o1, o[1], atol=2e-2)


def test_eligibility():
    w = torch.zeros(4, 4)
    assert is_muon_hidden_weight("backbone.0.encoder.layer.0.mlp.fc1.weight", w)
    assert is_muon_hidden_weight("backbone.0.encoder.layer.0.attention.qkv_weight", w)
    assert not is_muon_hidden_weight("class_embed.weight", w)
    assert not is_muon_hidden_weight("query_feat.weight", w)
    assert not is_muon_hidden_weight("x.bias", torch.zeros(4))
    assert not is_muon_hidden_weight("backbone.0.encoder.embeddings.patch_embeddings.weight", w)


def _literal_step(p, g, state, lr, wd, beta, is_muon, t):
    """Straight per-tensor statement of one update."""
    if is_muon:
        state["m"].lerp_(g, 1 - beta)
        u = g.lerp(state["m"], beta).reshape(g.shape[0], -1)
        o = newton_schulz5(u).float() * math.sqrt(max(1.0, u.shape[0] / u.shape[1]))
        p.mul_(1 - lr * wd).add_(o.view_as(p), alpha=-lr)
    else:
        state["a"].lerp_(g, 0.1)
        state["b"].lerp_(g * g, 0.05)
        upd = (state["a"] / (1 - 0.9 ** t)) / ((state["b"] / (1 - 0.95 ** t)).sqrt() + 1e-10)
        p.mul_(1 - lr * wd).add_(upd, alpha=-lr)


def test_step_matches_literal_statement():
    torch.manual_seed(1)
    names = ["l.fc1.weight", "l.fc2.weight", "l.fc1.bias", "l.attention.qkv_weight"]
    shapes = [(32, 16), (32, 16), (32,), (48, 16)]
    ps = [torch.randn(s) for s in shapes]
    ref = [p.clone() for p in ps]
    groups = [{"lr": 0.02, "weight_decay": 0.01}, {"lr": 0.01, "weight_decay": 0.0}]
    opt = MuonAux(names, ps, [0, 0, 1, 0], groups, momentum=0.9)
    st = [{"m": torch.zeros(s), "a": torch.zeros(s), "b": torch.zeros(s)} for s in shapes]
    for t in range(1, 4):
        gs = [torch.randn(s) for s in shapes]
        opt.step(gs, lr_scale=0.5)
        for i, (n, p, g) in enumerate(zip(names, ref, gs)):
            gi = [0, 0, 1, 0][i]
            lr, wd = groups[gi]["lr"] * 0.5, groups[gi]["weight_decay"]
            if n.endswith("qkv_weight"):
                # three independent 16x16 matrices
                for k in range(3):
                    sub = {"m": st[i]["m"][16 * k:16 * (k + 1)]}
                    _literal_step(p[16 * k:16 * (k + 1)], g[16 * k:16 * (k + 1)], sub, lr, wd, 0.9, True, t)
            else:
                _literal_step(p, g, st[i], lr, wd, 0.9, is_muon_hidden_weight(n, p), t)
    for a, b in zip(ps, ref):
        assert torch.allclose(a, b, atol=2e-3), (a - b).abs().max()


def test_state_roundtrip():
    ps = [torch.randn(8, 4), torch.randn(4)]
    opt = MuonAux(["a.weight", "a.bias"], ps, [0, 0], [{"lr": 0.1, "weight_decay": 0.0}])
    opt.step([torch.randn(8, 4), torch.randn(4)])
    d = opt.state_dict()
    opt2 = MuonAux(["a.weight", "a.bias"], [p.clone() for p in ps], [0, 0], [{"lr": 0.1, "weight_decay": 0.0}])
    opt2.load_state_dict(d)
    assert torch.equal(opt2.state[0]["momentum_buffer"], opt.state[0]["momentum_buffer"])
    assert opt2.state[1]["step"] == 1


def test_loop_with_muon_and_resume(tmp_path):
    from mmltk_b200.ckpt import load_native_checkpoint
    from mmltk_b200.config import TrainOptions, apply_recipe
    from mmltk_b200.data.compiler import compile_split
    from mmltk_b200.data.source import write_synthetic_source
    from mmltk_b200.train.loop import run_training
    root = tmp_path / "src"
    write_synthetic_source(str(root), splits=("train", "val"), images=4, size=(40, 40), classes=2, seed=3)
    tr = compile_split(str(root), str(tmp_path / "b"), "train", width=32, height=32)["path"]
    va = compile_split(str(root), str(tmp_path / "b"), "val", width=32, height=32)["path"]
    o = TrainOptions(train_compiled=tr, val_compiled=va, output_dir=str(tmp_path / "o"), preset="rf-detr-tiny-test",
                     batch_size=2, epochs=1, optimizer="muon", workers=1)
    apply_recipe(o)
    run_training(o)
    ck = load_native_checkpoint(str(tmp_path / "o" / "checkpoint.pt"))
    assert ck.extra["optimizer_kind"] == "muon" and ck.extra["optimizer"]["kind"] == "muon"
    o2 = TrainOptions(train_compiled=tr, val_compiled=va, output_dir=str(tmp_path / "o2"),
                      preset="rf-detr-tiny-test", batch_size=2, epochs=2, optimizer="muon", workers=1,
                      resume=str(tmp_path / "o" / "checkpoint.pt"))
    apply_recipe(o2)
    res = run_training(o2)
    assert res["last_epoch"] == 1


@pytest.mark.gpu
def test_muon_engine_gpu_steps():
    from mmltk_b200.config import TrainOptions, apply_recipe
    from mmltk_b200.data.synthetic import synthetic_batch
    from mmltk_b200.models.rfdetr import build_model
    from mmltk_b200.train.engine import TrainEngine
    torch.manual_seed(0)
    m = build_model("rf-detr-medium", group_detr=2, dec_layers=2)
    o = TrainOptions(batch_size=2, optimizer="muon", use_ema=True)
    apply_recipe(o)
    eng = TrainEngine(m, o, "cuda", max_targets=10, steps_per_epoch=10, total_steps=10)
    eng.bind_static_inputs(2, 3, 576, 576)
    x, t = synthetic_batch(2, 576, kmax=10, slots=10, dtype=torch.bfloat16)
    losses = [eng.step(x.cuda(), t.to("cuda")).loss for _ in range(3)]
    assert all(math.isfinite(v) for v in losses)
    d = eng.optimizer_state()
    assert d["kind"] == "muon" and d["step"] == 3
