"""
The tuned torch layers on a GPU: TunedLinear / TunedLayerNorm /
TunedMultiheadAttention compute with the kernel library and match torch's own
layers (fp64 references for the GEMM and LayerNorm, SDPA in fp32 on the same
bf16 inputs for attention), within the families' tolerances.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import tuned_modules as tm  # noqa: E402


def test_tuned_linear_and_layernorm(dev, lib):
    torch.manual_seed(0)
    x = torch.randn(3, 50, 256, device=dev)
    lin = torch.nn.Linear(256, 384).to(dev)
    tl = tm.TunedLinear(256, 384).to(dev)
    tl.load_state_dict(lin.state_dict())
    tf = tm.TunedLinear(256, 384, variant="ffma").to(dev)
    tf.load_state_dict(lin.state_dict())
    ln = torch.nn.LayerNorm(384).to(dev)
    with torch.no_grad():
        ln.weight.uniform_(0.5, 1.5)
        ln.bias.uniform_(-0.2, 0.2)
    tln = tm.TunedLayerNorm(384).to(dev)
    tln.load_state_dict(ln.state_dict())
    with torch.no_grad():
        want = (x.double() @ lin.weight.double().T + lin.bias.double())
        for layer, tol in ((tl, 1e-3), (tf, 1e-5)):
            got = layer(x)
            assert got.shape == want.shape
            assert float((got.double() - want).abs().max() / want.abs().max()) <= tol
        y = tl(x)
        got = tln(y)
        ref = torch.nn.functional.layer_norm(y.double(), (384,), ln.weight.double(), ln.bias.double(), 1e-5)
        assert float((got.double() - ref).abs().max() / ref.abs().max()) <= 1e-5
    with pytest.raises(RuntimeError):
        tl(x.requires_grad_())
    assert lib.device_error() == 0


@pytest.mark.parametrize("causal", [False, True])
def test_tuned_mha_matches_torch(dev, lib, causal):
    torch.manual_seed(1)
    E, H, S, B = 512, 4, 300, 2
    ref = torch.nn.MultiheadAttention(E, H, batch_first=True).to(dev).eval()
    mha = tm.TunedMultiheadAttention(E, H).to(dev).eval()
    w = ref.in_proj_weight.detach()
    b = ref.in_proj_bias.detach()
    with torch.no_grad():
        for i, proj in enumerate((mha.q_proj, mha.k_proj, mha.v_proj)):
            proj.weight.copy_(w[i * E:(i + 1) * E])
            proj.bias.copy_(b[i * E:(i + 1) * E])
        mha.out_proj.weight.copy_(ref.out_proj.weight)
        mha.out_proj.bias.copy_(ref.out_proj.bias)
        x = torch.randn(B, S, E, device=dev)
        mask = torch.ones(S, S, dtype=torch.bool, device=dev).triu(1) if causal else None
        want, _ = ref(x, x, x, attn_mask=mask, need_weights=False)
        got, _ = mha(x, x, x, is_causal=causal)
    err = float((got - want).abs().max() / want.abs().max())
    assert err <= 2e-2, err
    assert lib.device_error() == 0


@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_comparison(dev, lib, causal):
    r = tm.sdpa_comparison(batch=2, heads=4, seq_len=1024, head_dim=128, causal=causal, warmup=1, samples=3, lib=lib)
    assert r["normwise_diff"] <= 2e-2
    assert r["kt_ms"] > 0 and r["sdpa_ms"] > 0
