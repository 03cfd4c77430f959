"""Vision building blocks on CPU: config rules, patch embedding, bicubic position resampling, DropPath,
masked bidirectional attention, pixel shuffle, visual-mask packing, projector, placeholder composition,
and the Swin window helpers.

Oracles: the equations of ``src/vision/vision_attention.py:8-81`` (softmax over valid keys only),
``positional_embedding.py:12-62`` (identity at the base grid, bicubic otherwise), ``pixel_shuffle.py:10-37``
(each 2x2 neighbourhood becomes one 4D token), ``src/kimi_k3/multimodal_composer.py:11-178`` (placeholders
replaced in order, sequence length unchanged) and ``swin_encoder.py`` (window partition / merge).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.vision import (DropPath, LearnedAbsolutePositionEmbedding, MoonViTEncoder,
                                        SpatialTokenPixelShuffle, VisionEncoderConfig, VisionPatchEmbedding,
                                        VisionProjector, VisionSelfAttention, VisualPlaceholderComposer,
                                        pack_visual_mask)
from kimi_k3_b200.models.vision_ablations import window_merge, window_partition

F64 = torch.float64


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [dict(image_size=30, patch_size=14), dict(embed_dim=0), dict(num_heads=5),
                                 dict(mlp_ratio=0.0), dict(position_embedding_type="rope"), dict(dropout=1.0),
                                 dict(drop_path_rate=-0.1), dict(initializer_std=0.0)])
def test_config_rejects_invalid_values(bad):
    kw = dict(image_size=28, patch_size=14, embed_dim=16, depth=1, num_heads=4)
    kw.update(bad)
    with pytest.raises(ValueError):
        VisionEncoderConfig(**kw)


# --------------------------------------------------------------------------- patches and positions
def test_patch_embedding_is_a_linear_map_of_each_patch():
    torch.manual_seed(0)
    pe = VisionPatchEmbedding(3, 8, 4, bias=True).double()
    img = torch.randn(2, 3, 8, 12, dtype=F64)
    tokens, grid = pe(img)
    assert grid == (2, 3) and tokens.shape == (2, 6, 8)
    w = pe.projection.weight.reshape(8, -1)
    patch = img[:, :, 4:8, 8:12].reshape(2, -1)          # row 1, column 2 -> token 1 * 3 + 2
    assert max_diff(tokens[:, 5], patch @ w.T + pe.projection.bias) < 1e-12
    with pytest.raises(ValueError):
        pe(torch.randn(1, 3, 9, 12, dtype=F64))
    with pytest.raises(ValueError):
        pe(torch.randn(1, 4, 8, 12, dtype=F64))


def test_position_embedding_identity_on_base_grid_and_bicubic_elsewhere():
    torch.manual_seed(1)
    pos = LearnedAbsolutePositionEmbedding((3, 4), 5).double()
    assert max_diff(pos((3, 4)), pos.patch_positions) == 0.0
    grid = pos.patch_positions.reshape(1, 3, 4, 5).permute(0, 3, 1, 2)
    want = F.interpolate(grid, size=(6, 2), mode="bicubic", align_corners=False).permute(0, 2, 3, 1).reshape(1, 12, 5)
    assert max_diff(pos((6, 2)), want) < 1e-6
    with_cls = LearnedAbsolutePositionEmbedding((3, 4), 5, use_cls_token=True)
    out = with_cls((3, 4))
    assert out.shape == (1, 13, 5) and torch.equal(out[:, :1], with_cls.cls_position)


def test_drop_path_scales_kept_samples_and_is_identity_in_eval():
    dp = DropPath(0.5)
    x = torch.ones(4000, 3)
    dp.train()
    torch.manual_seed(2)
    y = dp(x)
    kept = y[:, 0] != 0
    assert torch.all((y[kept] == 2.0)) and abs(kept.float().mean().item() - 0.5) < 0.05
    assert torch.equal(y[:, 0], y[:, 1])                 # whole samples are kept or dropped
    dp.eval()
    assert torch.equal(dp(x), x)
    with pytest.raises(ValueError):
        DropPath(1.0)


# --------------------------------------------------------------------------- attention
def test_masked_attention_ignores_padded_keys():
    torch.manual_seed(3)
    att = VisionSelfAttention(8, 2).double()
    x = torch.randn(2, 6, 8, dtype=F64)
    mask = torch.ones(2, 6, dtype=torch.bool)
    mask[1, 4:] = False
    out, probs = att(x, mask, output_attentions=True)
    assert probs[1, :, :, 4:].abs().max().item() == 0.0
    assert max_diff(probs.sum(-1), torch.ones(2, 2, 6, dtype=F64)) < 1e-6
    # changing padded tokens does not change the valid tokens' outputs
    x2 = x.clone()
    x2[1, 4:] = torch.randn(2, 8, dtype=F64)
    out2, _ = att(x2, mask)
    assert max_diff(out2[1, :4], out[1, :4]) < 1e-12
    # the equation: softmax(q k^T / sqrt(d)) v over valid keys, then the projection
    qkv = att.qkv(x[0]).reshape(6, 3, 2, 4).permute(1, 2, 0, 3)
    p = torch.softmax(qkv[0] @ qkv[1].transpose(-1, -2) / 2.0, -1)
    want = att.projection((p @ qkv[2]).transpose(0, 1).reshape(6, 8))
    assert max_diff(out[0], want) < 1e-6  # the softmax runs in fp32


def test_encoder_is_permutation_equivariant_without_positions():
    torch.manual_seed(4)
    enc = MoonViTEncoder(VisionEncoderConfig(image_size=16, patch_size=4, embed_dim=16, depth=2, num_heads=4,
                                             position_embedding_type="none")).double().eval()
    img = torch.randn(1, 3, 16, 16, dtype=F64)
    out = enc(img).last_hidden_state
    # swapping two patch columns of the image swaps the matching tokens
    img2 = img.clone()
    img2[..., 0:4], img2[..., 8:12] = img[..., 8:12], img[..., 0:4]
    out2 = enc(img2).last_hidden_state.reshape(1, 4, 4, 16)
    ref_ = out.reshape(1, 4, 4, 16)
    assert max_diff(out2[:, :, 0], ref_[:, :, 2]) < 1e-5 and max_diff(out2[:, :, 2], ref_[:, :, 0]) < 1e-5
    hs = enc(img, output_hidden_states=True).hidden_states
    assert len(hs) == 3 and max_diff(hs[-1], out) == 0.0


# --------------------------------------------------------------------------- packing and projection
def test_pixel_shuffle_packs_2x2_neighbourhoods():
    tokens = torch.arange(2 * 4 * 6 * 3, dtype=F64).reshape(2, 24, 3)
    out = SpatialTokenPixelShuffle()(tokens, (4, 6))
    assert out.grid_size == (2, 3) and out.last_hidden_state.shape == (2, 6, 12)
    grid = tokens.reshape(2, 4, 6, 3)
    # packed token (1, 2) holds rows 2-3, columns 4-5 in the order (r,c), (r,c+1), (r+1,c), (r+1,c+1)
    want = torch.cat((grid[:, 2, 4], grid[:, 2, 5], grid[:, 3, 4], grid[:, 3, 5]), -1)
    assert torch.equal(out.last_hidden_state[:, 1 * 3 + 2], want)
    with pytest.raises(ValueError):
        SpatialTokenPixelShuffle()(tokens[:, :20], (4, 5))


def test_visual_mask_packing_keeps_fully_valid_neighbourhoods():
    mask = torch.ones(1, 4, 4, dtype=torch.bool)
    mask[0, 3, 3] = False
    packed = pack_visual_mask(mask.reshape(1, 16), (4, 4))
    assert packed.tolist() == [[True, True, True, False]]
    with pytest.raises(ValueError):
        pack_visual_mask(torch.ones(1, 12, dtype=torch.bool), (3, 4))


def test_projector_is_a_two_layer_mlp():
    torch.manual_seed(5)
    p = VisionProjector(12, 20, 8, activation="silu", bias=True).double()
    x = torch.randn(2, 3, 12, dtype=F64)
    want = p.fc2(F.silu(p.fc1(x)))
    assert max_diff(p(x), want) == 0.0
    with pytest.raises(ValueError):
        VisionProjector(12, 20, 8, activation="relu6")
    with pytest.raises(ValueError):
        p(torch.randn(2, 3, 11, dtype=F64))


# --------------------------------------------------------------------------- composition
def test_composer_replaces_placeholders_in_order():
    comp = VisualPlaceholderComposer(4, image_token_id=7, video_token_id=8)
    ids = torch.tensor([[1, 7, 7, 2, 7, 3], [7, 1, 2, 3, 0, 0]])
    attn = torch.tensor([[1, 1, 1, 1, 1, 1], [1, 1, 1, 1, 0, 0]], dtype=torch.bool)
    text = torch.zeros(2, 6, 4, dtype=F64)
    # three images: sample 0 has two (2 and 1 valid tokens), sample 1 has one (1 valid token)
    proj = torch.arange(3 * 2 * 4, dtype=F64).reshape(3, 2, 4) + 1
    pmask = torch.tensor([[True, True], [True, False], [False, True]])
    out, meta = comp(text, ids, attn, image_embeddings=proj, image_mask=pmask, image_counts=torch.tensor([2, 1]))
    assert out.shape == text.shape
    assert torch.equal(out[0, 1], proj[0, 0]) and torch.equal(out[0, 2], proj[0, 1])
    assert torch.equal(out[0, 4], proj[1, 0]) and torch.equal(out[1, 0], proj[2, 1])
    assert torch.equal(out[0, 0], text[0, 0])
    assert meta.image_token_counts.tolist() == [3, 1]
    assert meta.image_positions.tolist() == [[0, 1], [0, 2], [0, 4], [1, 0]]


def test_composer_contract_errors():
    comp = VisualPlaceholderComposer(4, image_token_id=7, video_token_id=None)
    ids = torch.tensor([[7, 1, 7]])
    attn = torch.ones(1, 3, dtype=torch.bool)
    text = torch.zeros(1, 3, 4)
    with pytest.raises(ValueError):
        comp(text, ids, attn)                                            # placeholders without images
    with pytest.raises(ValueError):
        comp(text, ids, attn, image_embeddings=torch.zeros(1, 1, 4), image_mask=torch.ones(1, 1, dtype=torch.bool))
    with pytest.raises(ValueError):
        comp(text, ids, torch.tensor([[True, True, False]]), image_embeddings=torch.zeros(1, 2, 4),
             image_mask=torch.ones(1, 2, dtype=torch.bool))              # placeholder inside padding
    with pytest.raises(ValueError):
        comp(text, torch.tensor([[1, 1, 1]]), attn, video_embeddings=torch.zeros(1, 1, 4))
    with pytest.raises(ValueError):
        VisualPlaceholderComposer.resolve_counts("image_counts", torch.tensor([2]), 1, 3, "cpu")
    assert VisualPlaceholderComposer.resolve_counts("image_counts", None, 2, 2, "cpu").tolist() == [1, 1]


# --------------------------------------------------------------------------- Swin windows
@pytest.mark.parametrize("h,w,ws", [(8, 8, 4), (6, 10, 4), (7, 7, 3)])
def test_window_partition_and_merge_round_trip(h, w, ws):
    x = torch.randn(2, h, w, 5)
    win, meta = window_partition(x, ws)
    hp, wp = math.ceil(h / ws) * ws, math.ceil(w / ws) * ws
    assert win.shape == (2 * (hp // ws) * (wp // ws), ws * ws, 5)
    assert torch.equal(window_merge(win, ws, meta), x)
    # the first window holds the top-left ws x ws block, row by row
    assert torch.equal(win[0].reshape(ws, ws, 5)[:min(ws, h), :min(ws, w)], x[0, :ws, :ws])


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("kind", ["hierarchical", "swin"])
def test_kimi_k3_with_ablation_encoders_matches_reference(kind):
    """The full model with the hierarchical or Swin encoder as its vision tower: logits, loss and a
    backward pass, against the reference model holding the same weights; the config round-trips."""
    import dataclasses
    ref()
    import src.vision.hierarchical_encoder as rh
    import src.vision.swin_encoder as rs
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as rcfg
    from src.kimi_k3_mini import KimiK3 as RK
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    from kimi_k3_b200.models.kimi_k3 import KimiK3Config, VisionProjectorConfig
    from kimi_k3_b200.models.vision_ablations import HierarchicalVisionConfig, SwinVisionConfig
    kw = dict(image_size=32, patch_size=4, embed_dims=(8, 16), num_heads=(2, 4))
    if kind == "hierarchical":
        ours_v, theirs_v = (HierarchicalVisionConfig(depths=(1, 1), **kw),
                            rh.HierarchicalVisionConfig(depths=(1, 1), **kw))
    else:
        ours_v = SwinVisionConfig(depths=(2, 2), window_size=2, **kw)
        theirs_v = rs.SwinVisionConfig(depths=(2, 2), window_size=2, **kw)
    base, rbase = kimi_k3_cpu_tiny_config(), rcfg()
    cfg = dataclasses.replace(base, vision=ours_v, vision_projector=VisionProjectorConfig(64, 32, 16))
    rc = dataclasses.replace(rbase, vision=theirs_v,
                             vision_projector=dataclasses.replace(rbase.vision_projector, input_dim=64))
    assert KimiK3Config.from_dict(cfg.to_dict()) == cfg
    torch.manual_seed(0)
    ours, theirs = KimiK3(cfg).double(), RK(rc).double()
    theirs.load_state_dict(ours.state_dict())
    img = torch.randn(1, 3, 32, 32, dtype=F64)
    ids = torch.randint(5, 128, (1, 12))
    ids[0, 2:6] = cfg.image_token_id          # 8x8 patches, one 2x pooling / merge, 2x2 shuffle -> 4 tokens
    a = ours(input_ids=ids, pixel_values=img, labels=ids, use_mtp=True)
    b = theirs(input_ids=ids, pixel_values=img, labels=ids, use_mtp=True)
    assert max_diff(a.logits, b.logits) < 1e-12 and abs(a.loss.item() - b.loss.item()) < 1e-12
    a.loss.backward()
    assert all(p.grad is not None for n, p in ours.named_parameters() if n.startswith("vision_encoder"))
