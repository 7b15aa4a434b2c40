"""Pins the oracle's vision tower and connector to the installed transformers SmolVLM modules (CPU).

The reference runs SmolVLA's embed_image through lerobot -> transformers (SmolVLMVisionTransformer +
SmolVLMConnector), which the reference does not ship; transformers 5.5 here ships both.  With identical
random bf16 weights and inputs:
  * patch embedding (+ position embedding), LayerNorm, the GELU(tanh) MLP, the post-LayerNorm, pixel shuffle
    and the modality projection are bit-exact;
  * attention agrees to cosine >= 0.9999: transformers' eager attention rounds Q.K^T to bf16 before its fp32
    softmax, while the oracle follows the reference's own restatement, which keeps the scores in fp32
    (deploy/export_6f_layer0_attention_tensors.py:100-119);
  * one encoder layer and the whole embed_image agree to cosine >= 0.9999 / 0.999.
A small vision configuration (64 px, 2 layers of width 128) keeps this to seconds.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle.model import OracleSmolVLA, layer_norm, pixel_shuffle
from smolvla_mujoco_libero_b200.config import CONNECTOR, TINY, VISION
from smolvla_mujoco_libero_b200.weights import random_weights

smolvlm = pytest.importorskip("transformers.models.smolvlm.modeling_smolvlm")
from transformers.models.smolvlm.configuration_smolvlm import SmolVLMConfig, SmolVLMVisionConfig  # noqa: E402

CFG = TINY.with_(image_size=64, vis_hidden=128, vis_heads=2, vis_mlp=256, vis_layers=2, scale_factor=2,
                 vocab=256, text_layers=1, expert_layers=1)


def cosine(a, b):
    return float(F.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0))


@pytest.fixture(scope="module")
def models():
    torch.manual_seed(0)
    w = random_weights(CFG, 11)
    vcfg = SmolVLMVisionConfig(hidden_size=CFG.vis_hidden, intermediate_size=CFG.vis_mlp,
                               num_hidden_layers=CFG.vis_layers, num_attention_heads=CFG.vis_heads,
                               num_channels=CFG.channels, image_size=CFG.image_size, patch_size=CFG.patch,
                               hidden_act="gelu_pytorch_tanh", layer_norm_eps=CFG.vis_eps)
    vcfg._attn_implementation = "eager"
    vision = smolvlm.SmolVLMVisionTransformer(vcfg).to(torch.bfloat16).eval()
    prefix = VISION + "."
    sd = {k[len(prefix):]: v for k, v in w.items() if k.startswith(prefix)}
    missing, unexpected = vision.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    mcfg = SmolVLMConfig(vision_config=vcfg.to_dict(), text_config={"hidden_size": CFG.hidden},
                         scale_factor=CFG.scale_factor)
    conn = smolvlm.SmolVLMConnector(mcfg).to(torch.bfloat16).eval()
    conn.load_state_dict({"modality_projection.proj.weight": w[f"{CONNECTOR}.weight"]})
    orc = OracleSmolVLA(CFG, w, mode="bf16")
    img = torch.rand(2, CFG.channels, CFG.image_size, CFG.image_size, generator=torch.Generator().manual_seed(3))
    return w, vision, conn, orc, img


@torch.no_grad()
def test_patch_embedding_is_bit_exact(models):
    w, vision, _, orc, img = models
    grid = CFG.image_size // CFG.patch
    ref = vision.embeddings(pixel_values=img.to(torch.bfloat16),
                            patch_attention_mask=torch.ones(2, grid, grid, dtype=torch.bool))
    assert torch.equal(orc.vision_embeddings(img), ref)


@torch.no_grad()
def test_encoder_layer_steps(models):
    w, vision, _, orc, img = models
    h = orc.vision_embeddings(img)
    layer = vision.encoder.layers[0]
    p = f"{VISION}.encoder.layers.0"
    y = layer_norm(h, w[f"{p}.layer_norm1.weight"], w[f"{p}.layer_norm1.bias"], CFG.vis_eps)
    assert torch.equal(y, layer.layer_norm1(h))
    y2 = layer_norm(h, w[f"{p}.layer_norm2.weight"], w[f"{p}.layer_norm2.bias"], CFG.vis_eps)
    assert torch.equal(y2, layer.layer_norm2(h))
    assert torch.equal(orc.vision_mlp(0, y2), layer.mlp(y2))          # fc1 -> GELU(tanh) -> fc2
    attn, _ = layer.self_attn(y)
    assert cosine(orc.vision_attention(0, y), attn) >= 0.9999
    assert cosine(orc.vision_layer(0, h), layer(h, attention_mask=None)) >= 0.9999


@torch.no_grad()
def test_post_layernorm_pixel_shuffle_and_connector_are_bit_exact(models):
    w, vision, conn, orc, img = models
    h = torch.randn(2, (CFG.image_size // CFG.patch) ** 2, CFG.vis_hidden).to(torch.bfloat16)
    post = layer_norm(h, w[f"{VISION}.post_layernorm.weight"], w[f"{VISION}.post_layernorm.bias"], CFG.vis_eps)
    assert torch.equal(post, vision.post_layernorm(h))
    assert torch.equal(pixel_shuffle(post, CFG.scale_factor), conn.pixel_shuffle(post, CFG.scale_factor))
    assert torch.equal(orc.connector(post), conn(post))
    # the benchmark's shape: 1024 patches of width 768, shuffled by 4
    big = torch.randn(2, 1024, 768).to(torch.bfloat16)
    assert torch.equal(pixel_shuffle(big, 4), conn.pixel_shuffle(big, 4))


@torch.no_grad()
def test_embed_image_against_transformers(models):
    w, vision, conn, orc, img = models
    ref = conn(vision(pixel_values=img.to(torch.bfloat16)).last_hidden_state)
    got = orc.embed_image(img)
    assert got.shape == ref.shape == (2, CFG.n_img_tokens, CFG.hidden)
    assert cosine(got, ref) >= 0.999
