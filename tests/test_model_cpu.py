"""Model structure, checkpoint key layout and numerics of the CPU (oracle) path."""
import math

import pytest
import torch

from mmltk_b200.config import config_from_preset, infer_preset_from_path, find_preset
from mmltk_b200.models import RFDETR, build_model
from mmltk_b200.models.transformer import encoder_proposals, gen_sineembed_for_position


def tiny(**kw):
    return build_model("rf-detr-tiny-test", **kw)


def test_state_dict_uses_reference_key_layout():
    m = build_model("rf-detr-nano")
    keys = set(m.state_dict().keys())
    must = [
        "backbone.0.encoder.encoder.embeddings.cls_token",
        "backbone.0.encoder.encoder.embeddings.position_embeddings",
        "backbone.0.encoder.encoder.embeddings.patch_embeddings.projection.weight",
        "backbone.0.encoder.encoder.encoder.layer.0.norm1.weight",
        "backbone.0.encoder.encoder.encoder.layer.0.attention.attention.query.weight",
        "backbone.0.encoder.encoder.encoder.layer.11.attention.attention.value.bias",
        "backbone.0.encoder.encoder.encoder.layer.3.attention.output.dense.weight",
        "backbone.0.encoder.encoder.encoder.layer.5.layer_scale1.lambda1",
        "backbone.0.encoder.encoder.encoder.layer.5.mlp.fc1.weight",
        "backbone.0.encoder.encoder.layernorm.weight",
        "backbone.0.projector.stages.0.0.cv1.conv.weight",
        "backbone.0.projector.stages.0.0.cv1.bn.weight",
        "backbone.0.projector.stages.0.0.m.2.cv2.conv.weight",
        "backbone.0.projector.stages.0.1.weight",
        "transformer.decoder.layers.0.self_attn.in_proj_weight",
        "transformer.decoder.layers.1.cross_attn.sampling_offsets.weight",
        "transformer.decoder.layers.1.cross_attn.value_proj.bias",
        "transformer.decoder.ref_point_head.layers.1.weight",
        "transformer.decoder.norm.weight",
        "transformer.enc_output.0.weight",
        "transformer.enc_output.12.bias",
        "transformer.enc_output_norm.7.weight",
        "transformer.enc_out_class_embed.3.weight",
        "transformer.enc_out_bbox_embed.12.layers.2.bias",
        "class_embed.weight", "bbox_embed.layers.2.weight", "refpoint_embed.weight", "query_feat.weight",
    ]
    for k in must:
        assert k in keys, k
    assert not any("qkv" in k for k in keys)
    assert m.state_dict()["refpoint_embed.weight"].shape == (3900, 4)


def test_state_dict_roundtrip_and_qkv_split():
    torch.manual_seed(0)
    a = tiny()
    b = tiny()
    sd = a.state_dict()
    b.load_state_dict(sd, strict=True)
    for k, v in b.state_dict().items():
        assert torch.equal(v, sd[k]), k
    layer = a.backbone[0].encoder.encoder.encoder.layer[0].attention.attention
    C = layer.width
    assert torch.equal(sd["backbone.0.encoder.encoder.encoder.layer.0.attention.attention.key.weight"],
                       layer.qkv_weight[C:2 * C])


def test_init_matches_reference_conventions():
    m = build_model("rf-detr-nano")
    prior = -math.log((1 - 0.01) / 0.01)
    assert torch.allclose(m.class_embed.bias, torch.full_like(m.class_embed.bias, prior))
    assert torch.allclose(m.transformer.enc_out_class_embed.bias, torch.full_like(m.transformer.enc_out_class_embed.bias,
                                                                                  prior))
    assert m.refpoint_embed.weight.abs().max() == 0
    assert m.bbox_embed.layers[2].weight.abs().max() == 0
    ca = m.transformer.decoder.layers[0].cross_attn
    assert ca.attention_weights.weight.abs().max() == 0
    # grid init: head 0 points along +x with magnitude (point index + 1)
    b = ca.sampling_offsets.bias.view(ca.n_heads, ca.n_levels, ca.n_points, 2)
    assert torch.allclose(b[0, 0, :, 0], torch.arange(1, ca.n_points + 1, dtype=torch.float32))


def test_forward_shapes_train_and_eval():
    torch.manual_seed(0)
    m = tiny(resolution=64)
    x = torch.randn(2, 3, 64, 64)
    m.train()
    o = m(x)
    Q = m.cfg.num_queries * m.cfg.group_detr
    assert o["pred_logits"].shape == (2, Q, m.cfg.num_classes)
    assert o["pred_boxes"].shape == (2, Q, 4)
    assert len(o["aux_outputs"]) == m.cfg.dec_layers - 1
    assert o["enc_outputs"]["pred_logits"].shape == (2, Q, m.cfg.num_classes)
    m.eval()
    with torch.no_grad():
        o = m(x)
    assert o["pred_logits"].shape == (2, m.cfg.num_queries, m.cfg.num_classes)


def test_windowing_is_a_permutation_of_tokens():
    """With identity layers the windowed backbone must return the un-windowed grid."""
    cfg = config_from_preset("rf-detr-tiny-test", num_windows=2, resolution=64, positional_encoding_size=4)
    m = RFDETR(cfg)
    enc = m.backbone[0].encoder.encoder
    for layer in enc.encoder.layer:
        layer.layer_scale1.lambda1.data.zero_()
        layer.layer_scale2.lambda1.data.zero_()
    enc.layernorm.weight.data.fill_(1.0)
    enc.layernorm.bias.data.zero_()
    x = torch.randn(2, 3, 64, 64)
    feats = enc(x)
    tokens = enc.embeddings.patch_embeddings(x) + enc.embeddings.position_embeddings[:, 1:]
    expect = torch.nn.functional.layer_norm(tokens, (cfg.vit_width,), eps=1e-6).view(2, 4, 4, -1)
    assert torch.allclose(feats[0], expect, atol=1e-5)


def test_proposals_and_sine_embedding():
    p, valid = encoder_proposals([(4, 5)], 1, "cpu", torch.float32, False)
    assert p.shape == (1, 20, 4)
    assert torch.allclose(p[0, 0], torch.tensor([0.1, 0.125, 0.05, 0.05]))
    e = gen_sineembed_for_position(torch.rand(3, 7, 4), 64)
    assert e.shape == (3, 7, 256)


def test_sine_embedding_matches_interleaved_sin_cos():
    """sin(v f + phase) form == the reference's interleaved sin / cos of (y, x, w, h)."""
    import math
    pos = torch.rand(2, 9, 4, dtype=torch.float64)
    dim = 64
    t = 10000.0 ** (2 * (torch.arange(dim, dtype=torch.float64) // 2) / dim)
    ref = []
    for c in (1, 0, 2, 3):
        x = pos[..., c, None] * 2 * math.pi / t
        ref.append(torch.stack((x[..., 0::2].sin(), x[..., 1::2].cos()), -1).flatten(-2))
    ref = torch.cat(ref, -1)
    got = gen_sineembed_for_position(pos, dim).double()
    assert torch.allclose(got, ref, atol=2e-6)


def test_preset_inference_from_paths():
    assert infer_preset_from_path("/w/rf-detr-medium.pth").name == "rf-detr-medium"
    assert infer_preset_from_path("/x/my_seg-2xl_run/checkpoint.pth").name == "rf-detr-seg-xxlarge"
    assert infer_preset_from_path("models/rf-detr-seg-m-ft.pth").name == "rf-detr-seg-medium"
    assert infer_preset_from_path("/tmp/large/weights.pth").name == "rf-detr-large"
    assert infer_preset_from_path("/tmp/nothing.pth") is None
    assert find_preset("rf-detr-base").patch_size == 14


def test_class_head_resize_repeats_rows():
    m = tiny()
    w = m.class_embed.weight.detach().clone()
    m.reinitialize_detection_head(w.shape[0] + 3)
    assert m.class_embed.weight.shape[0] == w.shape[0] + 3
    assert torch.equal(m.class_embed.weight[w.shape[0]:], w[:3])


def test_large_vitb_p3p5_builds():
    cfg = config_from_preset("rf-detr-large-vitb", resolution=128, positional_encoding_size=8, group_detr=1,
                             num_queries=20, num_select=20)
    m = RFDETR(cfg)
    m.eval()
    with torch.no_grad():
        o = m(torch.randn(1, 3, 128, 128))
    assert o["pred_boxes"].shape == (1, 20, 4)


def test_large_vitb_projector_layout_and_size():
    """Config 4: each backbone tap is resampled on its own (upstream ``stages_sampling[level][tap]``
    layout), which gives ~128 M parameters for ViT-B with P3 + P5."""
    cfg = config_from_preset("rf-detr-large-vitb")
    m = RFDETR(cfg)
    n = sum(p.numel() for p in m.parameters())
    assert abs(n - 128e6) / 128e6 < 0.05, n
    sd = m.state_dict()
    assert tuple(sd["backbone.0.projector.stages_sampling.0.3.0.weight"].shape) == (768, 384, 2, 2)
    assert tuple(sd["backbone.0.projector.stages_sampling.1.3.0.conv.weight"].shape) == (768, 768, 3, 3)
    assert tuple(sd["backbone.0.projector.stages.0.0.cv1.conv.weight"].shape)[1] == 4 * 384
    assert tuple(sd["backbone.0.projector.stages.1.0.cv1.conv.weight"].shape)[1] == 4 * 768
    # a P4-only model keeps the reference's layout: no sampling parameters at all
    med = RFDETR(config_from_preset("rf-detr-medium")).state_dict()
    assert not any("stages_sampling" in k for k in med)


def test_transposed_conv_as_gemm_matches_conv_transpose2d():
    from mmltk_b200.models.projector import TransposedConv2x
    torch.manual_seed(0)
    t = TransposedConv2x(12, 6)
    x = torch.randn(2, 5, 7, 12)
    ref = torch.nn.functional.conv_transpose2d(x.permute(0, 3, 1, 2), t.weight, t.bias, stride=2).permute(0, 2, 3, 1)
    assert torch.allclose(t.forward_nhwc(x), ref, atol=1e-5, rtol=1e-5)


def test_inference_encoder_path_matches_training_path():
    """Without autograd the ViT forms each LayerScale residual inside the next LayerNorm; the
    features must equal the autograd path's (random, non-trivial layer scales)."""
    torch.manual_seed(0)
    cfg = config_from_preset("rf-detr-tiny-test", num_windows=2, resolution=64, positional_encoding_size=4)
    m = RFDETR(cfg)
    enc = m.backbone[0].encoder.encoder
    for layer in enc.encoder.layer:
        layer.layer_scale1.lambda1.data.uniform_(0.2, 1.0)
        layer.layer_scale2.lambda1.data.uniform_(0.2, 1.0)
    x = torch.randn(2, 3, 64, 64)
    with torch.enable_grad():
        ref = [f.detach() for f in enc(x)]
    with torch.no_grad():
        got = enc(x)
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        assert torch.allclose(g, r, atol=1e-5, rtol=1e-5)


def test_scaled_residual_layer_norm_reference():
    from mmltk_b200.ops import scaled_residual_layer_norm
    torch.manual_seed(0)
    y, res = torch.randn(5, 7, 16), torch.randn(5, 7, 16)
    g, w, b = torch.rand(16), torch.randn(16), torch.randn(16)
    out, s = scaled_residual_layer_norm(y, res, g, w, b, 1e-6)
    assert torch.allclose(s, res + g * y)
    assert torch.allclose(out, torch.nn.functional.layer_norm(res + g * y, (16,), w, b, 1e-6), atol=1e-6)


def test_reparam_boxes_backward_matches_autograd():
    """The written-out backward of the box reparameterisation equals autograd's (float64 gradcheck
    plus a direct comparison against the slice-and-cat statement)."""
    from mmltk_b200.models.transformer import _ReparamBoxesFn, reparam_boxes
    torch.manual_seed(0)
    d = (0.3 * torch.randn(2, 5, 4, dtype=torch.float64)).requires_grad_()
    b = (0.2 + torch.rand(2, 5, 4, dtype=torch.float64)).requires_grad_()
    assert torch.autograd.gradcheck(_ReparamBoxesFn.apply, (d, b))
    g = torch.randn(2, 5, 4, dtype=torch.float64)
    out = reparam_boxes(d, b)
    gd, gb = torch.autograd.grad(out, (d, b), g)
    ref = torch.cat([d[..., :2] * b[..., 2:] + b[..., :2], d[..., 2:].exp() * b[..., 2:]], -1)
    rd, rb = torch.autograd.grad(ref, (d, b), g)
    assert torch.allclose(out, ref) and torch.allclose(gd, rd) and torch.allclose(gb, rb)
    bd = b.detach().requires_grad_()
    gb_only = torch.autograd.grad(reparam_boxes(d.detach(), bd), bd, g)[0]
    assert torch.allclose(gb_only, torch.autograd.grad(
        torch.cat([d.detach()[..., :2] * bd[..., 2:] + bd[..., :2], d.detach()[..., 2:].exp() * bd[..., 2:]], -1),
        bd, g)[0])
