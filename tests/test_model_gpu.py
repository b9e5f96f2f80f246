"""End-to-end mergenet_small_cls forward on the B200 kernels."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import carrier_mismatches
from oracle import routing as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


@torch.no_grad()
def torch_local_encoder(model, images):
    """Local blocks restated with PyTorch ops (band-masked softmax in fp32,
    conv patch embedding, exact GELU): x_embed [B, T, C] fp32."""
    w16 = model._weights16()
    cd = model.compute_dtype
    vit = model.local.vit
    b = images.shape[0]
    heads = model.num_heads
    x = F.conv2d(images.to(cd), w16["local.vit.patch_embed.proj.weight"], vit.patch_embed.proj.bias.to(cd),
                 stride=model.patch_size).flatten(2).transpose(1, 2)
    x = torch.cat([vit.cls_token.expand(b, -1, -1), x.float()], 1) + vit.pos_embed
    n, c = x.shape[1], x.shape[2]
    hd = c // heads
    pos = torch.arange(n, device=x.device)
    band = (pos[:, None] - pos[None, :]).abs() <= model.local_window
    band[0] = True
    for i, blk in enumerate(vit.blocks):
        h = F.layer_norm(x, (c,), blk.norm1.weight, blk.norm1.bias, blk.norm1.eps)
        qkv = model._linear16(h, f"local.vit.blocks.{i}.attn.qkv", blk.attn.qkv)
        q, k, v = qkv.view(b, n, 3, heads, hd).permute(2, 0, 3, 1, 4).unbind(0)
        s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(hd)
        a = torch.softmax(s.masked_fill(~band, float("-inf")), -1) @ v.float()
        a = a.to(cd).transpose(1, 2).reshape(b, n, c)
        x = x + model._linear16(a, f"local.vit.blocks.{i}.attn.proj", blk.attn.proj)
        h = F.layer_norm(x, (c,), blk.norm2.weight, blk.norm2.bias, blk.norm2.eps)
        h = F.gelu(model._linear16(h, f"local.vit.blocks.{i}.mlp.fc1", blk.mlp.fc1))
        x = x + model._linear16(h, f"local.vit.blocks.{i}.mlp.fc2", blk.mlp.fc2)
    return x


@torch.no_grad()
def torch_recovery(model, x_embed, topk_x):
    """MyCrossAttention + residual (model.py:122-221, :1193) restated with
    PyTorch ops as the reference runs it under fp16 autocast: fp32
    LayerNorms, IEEE fp32 q/k/v projections, attention on fp16 operands with
    an fp16 context, fp32 out-projection."""
    b, nq, c = topk_x.shape
    heads = model.num_heads
    hd = c // heads
    ca = model.encode_cross_attention
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        q = F.linear(F.layer_norm(topk_x, (c,), ca.q_norm.weight, ca.q_norm.bias), ca.q_proj.weight, ca.q_proj.bias)
        kv = F.layer_norm(x_embed, (c,), ca.kv_norm.weight, ca.kv_norm.bias)
        k = F.linear(kv, ca.k_proj.weight, ca.k_proj.bias)
        v = F.linear(kv, ca.v_proj.weight, ca.v_proj.bias)
        cd = model.compute_dtype
        split = lambda t: t.to(cd).view(b, -1, heads, hd).transpose(1, 2).float()  # noqa: E731
        ctx = torch.softmax(split(q) @ split(k).transpose(-1, -2) / math.sqrt(hd), -1) @ split(v)
        ctx = ctx.to(cd).float().transpose(1, 2).reshape(b, -1, c)  # SDPA's 16-bit output, widened
        return F.linear(ctx, ca.out_proj.weight, ca.out_proj.bias) + topk_x
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@torch.no_grad()
def torch_after_routing(model, x_trace, topk_size):
    """Six latent blocks with proportional attention and the head, restated
    with PyTorch ops from the recovery output (model.py:1195-1198)."""
    b, nq, c = x_trace.shape
    heads = model.num_heads
    hd = c // heads
    xt = x_trace
    log_size = topk_size.log().to(model.compute_dtype)[:, None, None, :]
    for i, blk in enumerate(model.latent.vit.blocks):
        # ToMeBlock with proportional attention (opentome/timm/tome.py:89-143)
        h = F.layer_norm(xt, (c,), blk.norm1.weight, blk.norm1.bias, blk.norm1.eps)
        qkv = model._linear16(h, f"latent.vit.blocks.{i}.attn.qkv", blk.attn.qkv)
        q, k, v = qkv.view(b, nq, 3, heads, hd).permute(2, 0, 3, 1, 4).unbind(0)
        a = F.scaled_dot_product_attention(q, k, v, attn_mask=log_size).transpose(1, 2).reshape(b, nq, c)
        xt = xt + model._linear16(a, f"latent.vit.blocks.{i}.attn.proj", blk.attn.proj)
        h = F.layer_norm(xt, (c,), blk.norm2.weight, blk.norm2.bias, blk.norm2.eps)
        h = F.gelu(model._linear16(h, f"latent.vit.blocks.{i}.mlp.fc1", blk.mlp.fc1))
        xt = xt + model._linear16(h, f"latent.vit.blocks.{i}.mlp.fc2", blk.mlp.fc2)
    lv = model.latent.vit
    cls = F.layer_norm(xt[:, 0], (c,), lv.norm.weight, lv.norm.bias, lv.norm.eps)
    tokens = F.layer_norm(xt[:, 1:], (c,), lv.norm.weight, lv.norm.bias, lv.norm.eps)
    return model._linear16(cls, "head", model.head), tokens


@torch.no_grad()
def live_out_proj(model, seed=0):
    """The reference zero-initialises the cross-attention out-projection
    (model.py:822-829), which would hide the recovery path from the logits;
    give it random weights so every check below sees it."""
    g = torch.Generator().manual_seed(seed)
    op = model.encode_cross_attention.out_proj
    op.weight.copy_(torch.randn(op.weight.shape, generator=g) * 0.05)
    op.bias.copy_(torch.randn(op.bias.shape, generator=g) * 0.05)
    model._reset_caches()
    return model


def check_forward(model, images, tol=1e-2, feat_tol=2e-3):
    """Stage-by-stage parity of one forward: local encoder vs the PyTorch
    restatement (fp16 tolerance), routing on the model's own x_embed/metrics
    vs the oracle (exact carriers), the recovery cross-attention output vs
    its fp32 restatement (2e-3, and large enough that a zeroed
    cross-attention would fail), logits vs the restatement of the latent
    stage fed with the model's recovery output (1e-2)."""
    logits, aux = model(images, return_intermediates=True)
    x_ref = torch_local_encoder(model, images)
    err = ((aux["x_embed"] - x_ref).abs().max() / x_ref.abs().max()).item()
    assert err <= tol, f"local encoder rel err {err}"
    x_np = aux["x_embed"].cpu().numpy()
    m_np = aux["metrics"].float().cpu().numpy()  # bf16 values are exact in float32
    route = O.route_and_gather(x_np, m_np, model.r_list, O.Geometry(model.grid, model.spatial_radius))
    mism = carrier_mismatches(aux["topk_patch_indices"].cpu().numpy(), route["topk_idx"], route["center"])
    assert not mism, mism
    rel = np.abs(aux["topk_x"].cpu().numpy() - route["topk_x"]).max() / np.abs(route["topk_x"]).max()
    assert rel <= feat_tol, rel
    rec = torch_recovery(model, aux["x_embed"], aux["topk_x"])
    scale = rec.abs().max()
    rerr = ((aux["x_trace"] - rec).abs().max() / scale).item()
    assert rerr <= feat_tol, f"recovery cross-attention rel err {rerr}"
    contrib = ((rec - aux["topk_x"]).abs().max() / scale).item()
    assert contrib >= 0.05, f"cross-attention contributes only {contrib} of the recovery output"
    exp, tokens = torch_after_routing(model, aux["x_trace"], aux["topk_size"])
    lerr = ((logits.float() - exp.float()).abs().max() / exp.float().abs().max()).item()
    assert lerr <= tol, f"logits rel err {lerr}"
    terr = ((aux["latent_tokens"] - tokens).abs().max() / tokens.abs().max()).item()
    assert terr <= tol, f"latent tokens rel err {terr}"
    return logits, aux


def test_reference_smoke_config(dev):
    """tests/test_model_smoke.py:27-134: a 32x32 model keeps 8 carriers and
    repeated eval forwards agree (here bit-exactly: no atomics anywhere)."""
    from mergenet_b200.model import MergeNetSmall
    torch.manual_seed(20260809)
    model = MergeNetSmall(img_size=32, patch_size=8, num_classes=10, metric_dim=16, local_depth=2,
                          latent_depth=2, local_window=2).init_weights(0)
    model = live_out_proj(model).to(dev).eval()
    images = torch.randn(2, 3, 32, 32, device=dev)
    first, aux1 = check_forward(model, images)
    second, aux2 = model(images)
    assert first.shape == (2, 10)
    assert aux1["retained_tokens"] == 8 == aux2["retained_tokens"]
    assert bool(torch.isfinite(first).all())
    assert torch.equal(first, second)


def test_canonical_forward_stages(dev):
    """Canonical 224x224 model, stage by stage."""
    from mergenet_b200.model import MergeNetSmall
    model = live_out_proj(MergeNetSmall().init_weights(0)).to(dev).eval()
    g = torch.Generator(device=dev).manual_seed(3)
    images = torch.randn(4, 3, 224, 224, device=dev, generator=g)
    logits, aux = check_forward(model, images)
    assert aux["retained_tokens"] == 392
    size = aux["token_strength_no_cls"].double().sum(1)
    torch.testing.assert_close(size, torch.full_like(size, 784.0), rtol=1e-5, atol=1e-3)


def test_forward_graph_replay_and_host_stream(dev):
    """The CUDA-graph forward equals the eager forward, and the overlapped
    host-batch path gives every batch its own logits."""
    from mergenet_b200.model import ForwardGraph, MergeNetSmall
    model = MergeNetSmall(img_size=32, patch_size=8, num_classes=10, metric_dim=16, local_depth=2,
                          latent_depth=2, local_window=2).init_weights(0).to(dev).eval()
    g = torch.Generator(device=dev).manual_seed(11)
    batches = [torch.randn(3, 3, 32, 32, device=dev, generator=g) for _ in range(3)]
    eager = [model(b)[0].clone() for b in batches]
    fwd = ForwardGraph(model, batches[0].clone(), warmup=1)
    for b, e in zip(batches, eager):
        got, _ = fwd(b)
        assert torch.equal(got, e)
    host = [b.cpu().pin_memory() for b in batches]
    out = torch.empty(3, 3, 10, dtype=eager[0].dtype).pin_memory()
    fwd.run_host_batches(host, out)
    torch.cuda.synchronize()
    for i, e in enumerate(eager):
        assert torch.equal(out[i], e.cpu())


def test_logits_match_the_reference_model(dev, golden_dir):
    """End to end against the reference's own model code: the fixture is the
    reference's mergenet_small_cls (its factory, LocalEncoder, DTEM merge
    loop, carrier block, cross-attention, ToMe latent blocks and head) run in
    fp32 on the host by make_model_golden.py, with stand-ins of this
    repository for timm's ViT modules and FlashAttention (neither is
    installed).  Here the same seeded weights load with strict=True and the
    forward runs on the B200 kernels under fp16 autocast semantics, so the
    tolerance is the fp16 one: logits and the CLS feature within 1e-2 of the
    largest magnitude.  The carriers are compared as sets: the fp16 metric
    heads round the scores, so sets may differ where the reference's masses
    are nearly tied."""
    from inputs import model_images, model_weights
    from mergenet_b200.model import mergenet_small_cls
    g = np.load(golden_dir / "model_small_cls.npz")
    shapes = {k: tuple(int(x) for x in v.split(",")) for k, v in zip(g["param_names"].tolist(),
                                                                       g["param_shapes"].tolist())}
    model = mergenet_small_cls()
    model.load_state_dict({k: torch.from_numpy(v) for k, v in model_weights(shapes, seed=0).items()}, strict=True)
    model = model.to(dev).eval()
    images = torch.from_numpy(model_images(0, int(g["batch"]))).to(dev)
    logits, aux = model(images)
    ref_logits = g["logits"]
    lerr = np.abs(logits.float().cpu().numpy() - ref_logits).max() / np.abs(ref_logits).max()
    ferr = rel(aux["cls_feature"].float().cpu().numpy(), g["cls_feature"])
    serr = rel(aux["token_strength_no_cls"].cpu().numpy(), g["token_strength_no_cls"])
    got, want = aux["topk_patch_indices"].cpu().numpy(), g["topk_patch_indices"]
    overlap = [len(set(got[b].tolist()) & set(want[b].tolist())) / want.shape[1] for b in range(want.shape[0])]
    print(f"logits rel {lerr:.2e}  cls rel {ferr:.2e}  masses rel {serr:.2e}  carrier overlap {overlap}")
    assert aux["retained_tokens"] == int(g["retained_tokens"])
    assert lerr <= 1e-2, lerr
    assert ferr <= 1e-2, ferr
    assert min(overlap) >= 0.97, overlap


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def test_high_resolution_bf16_forward(dev):
    """The 384 x 384, patch-8 configuration under bf16 autocast: a 48 x 48
    grid, 2305 tokens (windowed attention over 2305 tokens), 1152 carriers
    after six layers of 192 merges.  Stage by stage as above: the carriers
    on the model's own tokens and metrics equal the oracle's exactly, the
    rest within the bf16 tolerance (2e-2)."""
    from mergenet_b200.model import mergenet_small_cls
    model = live_out_proj(mergenet_small_cls(img_size=384, compute_dtype=torch.bfloat16).init_weights(0))
    model = model.to(dev).eval()
    assert model.grid == (48, 48) and model.r_list == [192] * 6
    g = torch.Generator(device=dev).manual_seed(5)
    images = torch.randn(2, 3, 384, 384, device=dev, generator=g)
    logits, aux = check_forward(model, images, tol=2e-2, feat_tol=2e-3)
    assert aux["retained_tokens"] == 1152
    assert aux["metrics"].dtype == torch.bfloat16
