"""Training loop end to end on CPU: outputs, checkpoints, resume, grad accumulation."""
import json
import os

import pytest
import torch

from mmltk_b200.ckpt import is_native_checkpoint, load_native_checkpoint
from mmltk_b200.config import TrainOptions
from mmltk_b200.data.compiler import compile_split
from mmltk_b200.data.source import write_synthetic_source
from mmltk_b200.train.loop import run_training


@pytest.fixture(scope="module")
def splits(tmp_path_factory):
    root = tmp_path_factory.mktemp("lsrc")
    write_synthetic_source(str(root), splits=("train", "val"), images=6, size=(48, 40), classes=3, seed=4)
    out = tmp_path_factory.mktemp("lbin")
    tr = compile_split(str(root), str(out), "train", width=32, height=32)["path"]
    va = compile_split(str(root), str(out), "val", width=32, height=32)["path"]
    return tr, va


def _opts(tr, va, out, **kw):
    o = TrainOptions(train_compiled=tr, val_compiled=va, output_dir=str(out), preset="rf-detr-tiny-test",
                     batch_size=2, epochs=2, workers=1, use_ema=True, seed=1)
    o.augmentation.enabled = True
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def test_train_outputs_and_resume(splits, tmp_path):
    tr, va = splits
    out = tmp_path / "run"
    res = run_training(_opts(tr, va, out))
    for f in ("checkpoint.pt", "checkpoint_epoch_1.pt", "checkpoint_epoch_2.pt", "checkpoint_best_regular.pt",
              "results.json", "log.txt", "progress.json", "eval_samples/epoch_0000.png",
              "eval_samples/epoch_0001.png"):
        assert os.path.exists(out / f), f
    assert open(out / "eval_samples" / "epoch_0000.png", "rb").read(8) == b"\x89PNG\r\n\x1a\n"
    assert is_native_checkpoint(str(out / "checkpoint.pt"))
    log = [json.loads(l) for l in open(out / "log.txt")]
    assert [r["epoch"] for r in log] == [0, 1]
    assert all(0 <= r["val"]["bbox"]["ap"] <= 1 for r in log) and "ap" in log[0]["ema_val"]["bbox"]
    prog = json.load(open(out / "progress.json"))
    assert prog["phase"] == "complete"
    results = json.load(open(out / "results.json"))
    assert results["last_epoch"] == 1 and results["history_size"] == 2 and res["best_checkpoint"]
    ck = load_native_checkpoint(str(out / "checkpoint.pt"))
    assert ck.extra["epoch"] == 1 and ck.extra["optimizer_kind"] == "adamw"
    assert ck.extra["optimizer"]["step"] == 2 * 3   # 3 batches of 2 per epoch
    assert "ema_state" in ck.extra and ck.metadata.preset_name == "rf-detr-tiny-test"
    # resume: one more epoch, optimizer step counter continues
    out2 = tmp_path / "resumed"
    res2 = run_training(_opts(tr, va, out2, resume=str(out / "checkpoint.pt"), epochs=3))
    log2 = [json.loads(l) for l in open(out2 / "log.txt")]
    assert [r["epoch"] for r in log2] == [2]
    assert load_native_checkpoint(str(out2 / "checkpoint.pt")).extra["optimizer"]["step"] == 9
    assert res2["last_epoch"] == 2


def test_resume_rejects_changed_schedule(splits, tmp_path):
    tr, va = splits
    out = tmp_path / "a"
    run_training(_opts(tr, va, out, epochs=1, use_ema=False))
    with pytest.raises(ValueError, match="lr_scheduler"):
        run_training(_opts(tr, va, tmp_path / "b", resume=str(out / "checkpoint.pt"), epochs=2,
                           lr_scheduler="cosine"))


def test_grad_accumulation_counts_optimizer_steps(splits, tmp_path):
    tr, va = splits
    out = tmp_path / "acc"
    run_training(_opts(tr, va, out, epochs=1, grad_accum_steps=3, use_ema=False))
    ck = load_native_checkpoint(str(out / "checkpoint.pt"))
    assert ck.extra["optimizer"]["step"] == 1


def test_validation_loss_and_profile(splits, tmp_path):
    tr, va = splits
    out = tmp_path / "vl"
    run_training(_opts(tr, va, out, epochs=1, use_ema=False, validation_loss=True, validation_profile=True,
                       print_freq=1))
    log = [json.loads(l) for l in open(out / "log.txt")]
    assert log[0]["val_loss"] is not None and log[0]["val_loss"] > 0
    prof = [json.loads(l) for l in open(out / "validation_profile.jsonl")]
    assert prof[0]["event"] == "rfdetr.validation.pass" and prof[0]["model_source"] == "regular"
