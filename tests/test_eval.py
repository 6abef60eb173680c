"""COCO evaluator against an independent Python statement of the same metric."""
import random

import pytest
import torch

from mmltk_b200.data.compiler import compile_split
from mmltk_b200.data.loader import CompiledDataset
from mmltk_b200.data.source import write_synthetic_source
from mmltk_b200.eval import CocoEvaluator

THR = [0.5 + 0.05 * t for t in range(10)]


def _iou(a, b):
    iw = max(0.0, min(a[2], b[2]) - max(a[0], b[0]))
    ih = max(0.0, min(a[3], b[3]) - max(a[1], b[1]))
    inter = iw * ih
    u = (a[2] - a[0]) * (a[3] - a[1]) + (b[2] - b[0]) * (b[3] - b[1]) - inter
    return 0.0 if u <= 0 else inter / u


def oracle_ap(gt, preds, ncls):
    """gt: {img: [(cls, box)]}; preds: {img: [(score, cls, box)]} (already capped)."""
    per_t = []
    for t in THR:
        aps = []
        for c in range(ncls):
            total = sum(1 for g in gt.values() for k, _ in g if k == c)
            if total == 0:
                continue
            recs = []
            for img, ps in preds.items():
                gts = [(o, b) for o, (k, b) in enumerate(gt.get(img, [])) if k == c]
                used = set()
                mine = sorted([(s, o, b) for o, (s, k, b) in enumerate(ps) if k == c], key=lambda x: -x[0])
                for s, o, b in mine:
                    best, bo = None, None
                    for go, gb in gts:
                        if go in used:
                            continue
                        v = float(torch.tensor(_iou(b, gb), dtype=torch.float32))
                        if v >= t and (best is None or v > best or (v == best and go < bo)):
                            best, bo = v, go
                    if bo is not None:
                        used.add(bo)
                    recs.append((s, img, o, bo is not None))
            recs.sort(key=lambda r: (-r[0], r[1], r[2]))
            tp, prec, rec = 0, [], []
            for i, r in enumerate(recs):
                tp += r[3]
                prec.append(tp / (i + 1))
                rec.append(tp / total)
            for i in range(len(prec) - 2, -1, -1):
                prec[i] = max(prec[i], prec[i + 1])
            ap = 0.0
            for k in range(101):
                idx = next((i for i, r in enumerate(rec) if r >= k * 0.01), None)
                if idx is not None:
                    ap += prec[idx]
            aps.append(ap / 101)
        per_t.append(sum(aps) / len(aps))
    return sum(per_t) / 10, per_t[0], per_t[5]


@pytest.fixture(scope="module")
def ds(tmp_path_factory):
    root = tmp_path_factory.mktemp("evsrc")
    write_synthetic_source(str(root), splits=("val",), images=10, size=(64, 64), classes=3, max_instances=4, seed=9)
    st = compile_split(str(root), str(tmp_path_factory.mktemp("evbin")), "val", width=64, height=64)
    return CompiledDataset(st["path"])


def _gt(ds):
    out = {}
    for i in range(len(ds)):
        b, c, _ = ds.instances(i)
        out[i] = [(int(k), [float(v) for v in bb]) for k, bb in zip(c.tolist(), b.tolist())]
    return out


def test_perfect_predictions_score_one(ds):
    gt = _gt(ds)
    ev = CocoEvaluator(ds)
    K = 6
    for i in range(len(ds)):
        g = gt[i]
        s = torch.zeros(1, K)
        lab = torch.full((1, K), -1, dtype=torch.int64)
        bx = torch.zeros(1, K, 4)
        for k, (c, b) in enumerate(g):
            s[0, k] = 0.9 - 0.01 * k
            lab[0, k] = c
            bx[0, k] = torch.tensor(b)
        ev.add([i], s, lab, bx)
    m = ev.summarize()["bbox"]
    assert m["ap"] == pytest.approx(1.0) and m["ap50"] == pytest.approx(1.0)


def test_matches_python_oracle(ds):
    gt = _gt(ds)
    rnd = random.Random(0)
    ev = CocoEvaluator(ds, max_dets=5)
    preds = {}
    K = 7
    for i in range(len(ds)):
        rows = []
        for k in range(K):
            if gt[i] and rnd.random() < 0.6:
                c, b = rnd.choice(gt[i])
                b = [v + rnd.uniform(-6, 6) for v in b]
                if rnd.random() < 0.2:
                    c = rnd.randrange(4)
            else:
                x, y = rnd.uniform(0, 50), rnd.uniform(0, 50)
                b, c = [x, y, x + rnd.uniform(3, 14), y + rnd.uniform(3, 14)], rnd.randrange(4)
            rows.append((round(rnd.random(), 3), c, b))
        rows.sort(key=lambda r: -r[0])
        kept, n = [], 0
        for r in rows:                       # the evaluator keeps the first max_dets valid labels
            if 0 <= r[1] < 4 and n < 5:
                kept.append(r)
                n += 1
        preds[i] = kept
        ev.add([i], torch.tensor([[r[0] for r in rows]]), torch.tensor([[r[1] for r in rows]]),
               torch.tensor([[r[2] for r in rows]]))
    m = ev.summarize()["bbox"]
    ap, ap50, ap75 = oracle_ap(gt, preds, 4)
    assert m["ap"] == pytest.approx(ap, abs=1e-9)
    assert m["ap50"] == pytest.approx(ap50, abs=1e-9) and m["ap75"] == pytest.approx(ap75, abs=1e-9)
    assert 0 < m["ap"] < 1


def test_export_import_equals_single_pass(ds):
    gt = _gt(ds)
    full = CocoEvaluator(ds)
    a, b = CocoEvaluator(ds), CocoEvaluator(ds)
    for i in range(len(ds)):
        s = torch.rand(1, 3)
        lab = torch.randint(0, 4, (1, 3))
        bx = torch.tensor([[gt[i][0][1] if gt[i] else [1.0, 1, 9, 9]] * 3])
        full.add([i], s, lab, bx)
        (a if i % 2 else b).add([i], s, lab, bx)
    a.ev.import_matches(b.ev.export_matches(False), False)
    assert a.summarize() == full.summarize()


def test_mask_ap_perfect(ds):
    gt = _gt(ds)
    ev = CocoEvaluator(ds, masks=True)
    for i in range(len(ds)):
        n = len(gt[i])
        if n == 0:
            ev.add([i], torch.zeros(1, 1), torch.full((1, 1), -1), torch.zeros(1, 1, 4), torch.zeros(1, 1, 64, 64))
            continue
        m = ds.masks([i], 100)[None]
        ev.add([i], torch.linspace(0.9, 0.5, n)[None], torch.tensor([[c for c, _ in gt[i]]]),
               torch.tensor([[b for _, b in gt[i]]]), m)
    out = ev.summarize()
    assert out["segm"]["ap"] == pytest.approx(1.0) and out["bbox"]["ap"] == pytest.approx(1.0)
