"""Fused row operations of include/mi_layers.h against the reference model's PyTorch chains.

Each kernel keeps the chain's rounding points, so the only freedom is the order of the fp32 sum
inside RMSNorm statistics (a few ulp of the statistic).  Hence:

* residual sums and SiLU*mul are bit-identical to PyTorch;
* RMSNorm / QK-norm+RoPE outputs: bit-identical for >= 99% of the elements in 16-bit types, the
  rest within one unit in the last place (of the element; for RoPE, whose two rounded terms can
  cancel, of the head's largest element); fp32 within 1e-6 relative;
* the decode append writes exactly the roped K and the raw V at the slots; a bad slot is
  skipped and reported in the status word;
* a fused model forward matches the reference's unfused chain (same weights) within the bf16
  attention tolerance.
"""

import pytest
import torch
import torch.nn.functional as F

from mini_infra_b200 import ops
from mini_infra_b200.model import Qwen3Config, build_model
from mini_infra_b200.model.config import TINY_C1

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def ref_rmsnorm(x, w, eps):  # reference model/qwen3.py:67-78
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(x.dtype)


def ref_rope(x, cos, sin):  # reference :112-144 (rotate-half)
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def assert_rounding_close(got, want, per_row=False):
    """>= 99% bit-identical; the rest within one unit in the last place of the element (per_row:
    of the row's largest element, for RoPE sums whose two rounded terms can cancel)."""
    if got.dtype == torch.float32:
        torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)
        return
    same = (got == want).float().mean().item()
    assert same >= 0.99, same
    eps = 2.0**-7 if got.dtype == torch.bfloat16 else 2.0**-10
    mag = want.float().abs()
    if per_row:
        mag = mag.amax(dim=-1, keepdim=True).expand_as(mag)
    ulp = torch.where(mag == 0, torch.ones_like(mag), mag) * eps
    assert ((got.float() - want.float()).abs() <= ulp * 1.01).all()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,hidden", [(1, 1024), (37, 1024), (300, 128), (5, 2560), (9, 4096), (4, 100)])
def test_rmsnorm_matches_reference(dtype, rows, hidden):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + hidden)
    x = torch.randn(rows, hidden, generator=g, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device="cuda")).to(dtype)
    assert_rounding_close(ops.rmsnorm(x, w, 1e-6), ref_rmsnorm(x, w, 1e-6))


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_with_residual_add(dtype):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(3, 17, 1024, generator=g, device="cuda").to(dtype)
    r = torch.randn(3, 17, 1024, generator=g, device="cuda").to(dtype)
    w = torch.randn(1024, generator=g, device="cuda").to(dtype)
    want_sum = r + x
    want = ref_rmsnorm(want_sum, w, 1e-6)
    r_in = r.clone()
    got = ops.rmsnorm(x, w, 1e-6, residual=r_in)
    assert torch.equal(r_in, want_sum)  # the residual add is one rounding, bit-exact
    assert_rounding_close(got, want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("cols", [3072, 384, 50])
def test_silu_mul_bit_exact(dtype, cols):
    g = torch.Generator(device="cuda").manual_seed(cols)
    gu = (3 * torch.randn(29, 2 * cols, generator=g, device="cuda")).to(dtype)
    gate, up = gu[:, :cols], gu[:, cols:]  # two halves of one GEMM output (shared row stride)
    assert torch.equal(ops.silu_mul(gate, up), F.silu(gate) * up)


def _qkv(tokens, hq, hkv, d, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    packed = torch.randn(tokens, (hq + 2 * hkv) * d, generator=g, device="cuda").to(dtype)
    q, k, v = packed[:, : hq * d], packed[:, hq * d : (hq + hkv) * d], packed[:, (hq + hkv) * d :]
    qw = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype)
    kw = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype)
    pos = torch.randint(0, 30000, (tokens,), generator=g, device="cuda")
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32, device="cuda") / d))
    ang = pos.float()[:, None] * inv_freq
    emb = torch.cat((ang, ang), dim=-1)
    return q, k, v, qw, kw, emb.cos().to(dtype), emb.sin().to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("d", [32, 64, 128, 256])
def test_qk_norm_rope_matches_reference(dtype, d):
    tokens, hq, hkv = 45, 8, 2
    q, k, v, qw, kw, cos, sin = _qkv(tokens, hq, hkv, d, dtype, d)
    q_out, k_out, v_out = ops.qk_norm_rope(q, k, v, qw, kw, cos, sin, 1e-6, hq, hkv)
    c, s = cos[:, None, :], sin[:, None, :]
    want_q = ref_rope(ref_rmsnorm(q.reshape(tokens, hq, d), qw, 1e-6), c, s)
    want_k = ref_rope(ref_rmsnorm(k.reshape(tokens, hkv, d), kw, 1e-6), c, s)
    assert_rounding_close(q_out, want_q, per_row=True)
    assert_rounding_close(k_out, want_k, per_row=True)
    assert torch.equal(v_out, v.reshape(tokens, hkv, d))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_qk_norm_rope_decode_append(dtype):
    tokens, hq, hkv, d, bs, nb = 12, 16, 8, 128, 16, 9
    q, k, v, qw, kw, cos, sin = _qkv(tokens, hq, hkv, d, dtype, 3)
    k_pool = torch.zeros(nb, bs, hkv, d, dtype=dtype, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    slots = torch.randperm(nb * bs - bs, device="cuda")[:tokens] + bs  # never the null block
    ops.read_status()
    q_out, k_none, _ = ops.qk_norm_rope(q, k, v, qw, kw, cos, sin, 1e-6, hq, hkv, kv_out=False,
                                        slot_mapping=slots, k_pool=k_pool, v_pool=v_pool)
    assert k_none is None
    _, k_ref, v_ref = ops.qk_norm_rope(q, k, v, qw, kw, cos, sin, 1e-6, hq, hkv)
    assert torch.equal(k_pool.view(-1, hkv, d)[slots], k_ref)
    assert torch.equal(v_pool.view(-1, hkv, d)[slots], v_ref)
    written = torch.zeros(nb * bs, dtype=torch.bool, device="cuda")
    written[slots] = True
    assert not k_pool.view(-1, hkv, d)[~written].any()
    assert ops.read_status() == 0
    bad = slots.clone()
    bad[3] = nb * bs  # one past the pool: skipped, reported
    before = k_pool.clone()
    ops.qk_norm_rope(q, k, v, qw, kw, cos, sin, 1e-6, hq, hkv, kv_out=False, slot_mapping=bad, k_pool=k_pool,
                     v_pool=v_pool)
    assert ops.read_status() == ops.nat.MI_STATUS_BAD_SLOT
    assert torch.equal(k_pool, before)  # same values rewritten at the good slots, nothing else


def _reference_forward(model, ids, pos):
    """The reference's unfused decoder chain on the same weights (prefill without history)."""
    m = model.model
    h = m.embed_tokens(ids)
    cos, sin = m.rotary_emb(pos, h.dtype)
    c, s = cos.unsqueeze(2), sin.unsqueeze(2)
    b, length, _ = h.shape
    for layer in m.layers:
        at = layer.self_attn
        x = ref_rmsnorm(h, layer.input_layernorm.weight, layer.input_layernorm.eps)
        q = ref_rope(ref_rmsnorm(F.linear(x, at.q_proj.weight).view(b, length, at.num_heads, -1), at.q_norm.weight, 1e-6), c, s)
        k = ref_rope(ref_rmsnorm(F.linear(x, at.k_proj.weight).view(b, length, at.num_kv_heads, -1), at.k_norm.weight, 1e-6), c, s)
        v = F.linear(x, at.v_proj.weight).view(b, length, at.num_kv_heads, -1)
        rep = at.num_heads // at.num_kv_heads
        qt, kt, vt = q.transpose(1, 2).float(), k.transpose(1, 2).repeat_interleave(rep, 1).float(), v.transpose(1, 2).repeat_interleave(rep, 1).float()
        scores = qt @ kt.transpose(-1, -2) * at.scaling
        mask = torch.ones(length, length, dtype=torch.bool, device=h.device).tril()
        probs = scores.masked_fill(~mask, float("-inf")).softmax(-1)
        attn = (probs @ vt).to(h.dtype).transpose(1, 2).reshape(b, length, -1)
        h = h + F.linear(attn, at.o_proj.weight)
        y = ref_rmsnorm(h, layer.post_attention_layernorm.weight, 1e-6)
        h = h + F.linear(F.silu(F.linear(y, layer.mlp.gate_proj.weight)) * F.linear(y, layer.mlp.up_proj.weight),
                         layer.mlp.down_proj.weight)
    return ref_rmsnorm(h, m.norm.weight, 1e-6)


@torch.inference_mode()
def test_fused_model_forward_matches_unfused_chain():
    cfg = Qwen3Config(**dict(TINY_C1, head_dim=128, hidden_size=256), torch_dtype="bfloat16")
    model = build_model(cfg, seed=11, device="cuda", dtype=torch.bfloat16)
    attn = model.model.layers[0].self_attn
    assert attn.q_proj.weight.data_ptr() == attn.packed_qkv.data_ptr()  # packed: one QKV GEMM
    g = torch.Generator(device="cuda").manual_seed(2)
    ids = torch.randint(0, cfg.vocab_size, (3, 40), generator=g, device="cuda")
    pos = torch.arange(40, device="cuda").expand(3, -1)
    hidden, _ = model.model(ids, position_ids=pos)
    want = _reference_forward(model, ids, pos)
    assert (hidden.float() - want.float()).abs().max().item() < 0.1 * want.float().abs().max().item()
    assert ops.read_status() == 0
