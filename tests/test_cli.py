"""Command line: compile / info / train (single and 2-rank gloo) / predict /
evaluate / export-onnx / normalize-weights, and the unavailable backends."""
import json
import os

import pytest

from mmltk_b200.cli.main import main
from mmltk_b200.data.source import write_synthetic_source


@pytest.fixture(scope="module")
def data(tmp_path_factory):
    root = tmp_path_factory.mktemp("csrc")
    write_synthetic_source(str(root), splits=("train", "val"), images=8, size=(40, 40), classes=2, seed=2)
    out = tmp_path_factory.mktemp("cbin")
    assert main(["compile", "--source", str(root), "--output", str(out), "--resolution", "32"]) == 0
    return out


def test_info_and_compile(data, capsys):
    assert main(["info", str(data / "train.bin")]) == 0
    h = json.loads(capsys.readouterr().out)
    assert h["num_images"] == 8 and h["width"] == 32


def test_train_predict_evaluate_export(data, tmp_path, capsys):
    out = tmp_path / "run"
    argv = ["rfdetr", "train", "--train-compiled", str(data / "train.bin"), "--val-compiled", str(data / "val.bin"),
            "--output-dir", str(out), "--preset", "rf-detr-tiny-test", "--batch-size", "2", "--epochs", "1",
            "--gpu-augment", "--aug-copy-paste-prob", "0.3", "--no-ema", "--workers", "1", "--compile-mode", "none"]
    assert main(argv) == 0
    best = json.loads(capsys.readouterr().out.strip().splitlines()[-1])["best_checkpoint"]
    assert os.path.exists(best)
    pred = tmp_path / "p.json"
    assert main(["rfdetr", "predict", "--compiled", str(data / "val.bin"), "--weights", best, "--output", str(pred),
                 "--threshold", "0.0", "--batch-size", "2"]) == 0
    js = json.load(open(pred))
    assert js["preset_name"] == "rf-detr-tiny-test" and len(js["records"]) == 8
    capsys.readouterr()
    assert main(["rfdetr", "evaluate", "--compiled", str(data / "val.bin"), "--weights", best]) == 0
    assert "bbox_ap=" in capsys.readouterr().out
    onnx = tmp_path / "m.onnx"
    assert main(["rfdetr", "export-onnx", "--weights", best, "--output", str(onnx)]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["opset"] == 19 and info["inputs"][0]["name"] == "input" and info["num_queries"] == 10
    norm = tmp_path / "n.pt"
    assert main(["rfdetr", "normalize-weights", "--input", best, "--output", str(norm)]) == 0
    assert main(["rfdetr", "info", str(norm)]) == 0
    assert main(["rfdetr", "build-engine", "--onnx", str(onnx), "--output", str(tmp_path / "e.plan")]) == 2
    assert main(["rfdetr", "predict", "--compiled", str(data / "val.bin"), "--onnx", str(onnx), "--output",
                 str(tmp_path / "x.json")]) == 2


def test_train_two_rank_gloo(data, tmp_path, monkeypatch):
    # CPU ranks over gloo, also on a machine with fewer GPUs than ranks: the children see no GPU
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    out = tmp_path / "ddp"
    argv = ["rfdetr", "train", "--train-compiled", str(data / "train.bin"), "--val-compiled", str(data / "val.bin"),
            "--output-dir", str(out), "--preset", "rf-detr-tiny-test", "--batch-size", "2", "--epochs", "1",
            "--device-ids", "0,1", "--workers", "2", "--compile-mode", "none"]
    assert main(argv) == 0
    log = [json.loads(l) for l in open(out / "log.txt")]
    assert len(log) == 1 and log[0]["effective_batch_global"] == 4
    assert os.path.exists(out / "checkpoint.pt")


def test_train_requires_inputs(data, tmp_path):
    with pytest.raises(SystemExit):
        main(["rfdetr", "train", "--train-compiled", str(data / "train.bin"), "--output-dir", str(tmp_path)])


def test_predict_draw_and_live(data, tmp_path, capsys):
    out = tmp_path / "draw"
    assert main(["rfdetr", "predict", "--compiled", str(data / "val.bin"), "--preset", "rf-detr-tiny-test",
                 "--output", str(tmp_path / "p.json"), "--threshold", "0.0", "--draw-dir", str(out)]) == 0
    assert len(list(out.glob("*.png"))) == 8
    capsys.readouterr()
    assert main(["rfdetr", "live", "--preset", "rf-detr-tiny-test", "--frames", "4", "--width", "64",
                 "--height", "48", "--threshold", "0.0"]) == 0
    st = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert st["frames_in"] == 4 and st["frames_analyzed"] >= 1
