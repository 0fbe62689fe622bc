"""GPU parity of the flash-attention forward (through the C-ABI) against the CPU oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import ATOL, RTOL, load_golden
from oracle import attention_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def run(pkg, q, k, v, causal, scale=None):
    out = pkg.flash_attn(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal, scale=scale)
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    return out.cpu()


@pytest.mark.parametrize("case", ["gqa", "mqa"])
@pytest.mark.parametrize("causal", [True, False])
def test_golden_fixture(cuda_pkg, case, causal):
    g = load_golden("attention")
    out = run(cuda_pkg, g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"], causal)
    want = g[f"{case}_out_{'causal' if causal else 'full'}"]
    torch.testing.assert_close(out.float(), want.float(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("case", ["gqa", "mqa"])
def test_golden_prompt_model(cuda_pkg, case):
    g = load_golden("attention")
    out = run(cuda_pkg, g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"], True,
              scale=attention_oracle.SM_SCALE_D128)
    torch.testing.assert_close(out.float(), g[f"{case}_out_model_causal"].float(), rtol=RTOL, atol=ATOL)


# ragged sequence lengths (not multiples of the 128-row tiles or the 256-row tile pairs),
# one-token and one-tile sequences, MHA / GQA / MQA head layouts
CASES = [
    (1, 1, 1, 1), (1, 7, 2, 2), (2, 128, 4, 2), (1, 129, 2, 1), (1, 256, 2, 2), (1, 257, 4, 4),
    (2, 300, 8, 2), (1, 384, 2, 1), (1, 640, 4, 1), (1, 1000, 8, 8), (2, 512, 8, 1), (1, 2048, 4, 2),
]


@pytest.mark.parametrize("B,S,Hq,Hkv", CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_matches_oracle(cuda_pkg, B, S, Hq, Hkv, causal):
    q, k, v = attention_oracle.attention_inputs(B, S, Hq, Hkv, 128, 20260314 + S)
    out = run(cuda_pkg, q, k, v, causal)
    want = attention_oracle.attention_reference(q, k, v, causal=causal)
    torch.testing.assert_close(out.float(), want.float(), rtol=RTOL, atol=ATOL)


def test_large_score_range_exercises_rescale(cuda_pkg):
    """Scores that grow along the sequence force the running maximum up many times."""
    q, k, v = attention_oracle.attention_inputs(1, 1024, 2, 1, 128, 5)
    ramp = torch.linspace(0.2, 6.0, 1024).view(1, 1024, 1, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    out = run(cuda_pkg, q, k, v, False)
    want = attention_oracle.attention_reference(q, k, v, causal=False)
    torch.testing.assert_close(out.float(), want.float(), rtol=RTOL, atol=ATOL)


def test_uniform_values_give_the_mean(cuda_pkg):
    """With V constant along the sequence the output equals V whatever the scores are."""
    q, k, v = attention_oracle.attention_inputs(1, 700, 4, 2, 128, 9)
    v = v[:, :1].expand(-1, 700, -1, -1).contiguous()
    out = run(cuda_pkg, q, k, v, True)
    want = v.float().repeat_interleave(2, dim=2)
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=1e-2)


def test_caller_owned_output_and_errors(cuda_pkg):
    q, k, v = attention_oracle.attention_inputs(1, 130, 2, 1, 128, 11)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.zeros_like(qd)
    ret = cuda_pkg.flash_attn(qd, kd, vd, causal=True, out=out)
    torch.cuda.synchronize()
    assert ret.data_ptr() == out.data_ptr()
    want = attention_oracle.attention_reference(q, k, v, causal=True)
    torch.testing.assert_close(out.cpu().float(), want.float(), rtol=RTOL, atol=ATOL)
    with pytest.raises(TypeError):
        cuda_pkg.flash_attn(qd, kd, vd, out=out.float())
    with pytest.raises(ValueError):
        cuda_pkg.flash_attn(qd[..., :64].contiguous(), kd[..., :64].contiguous(), vd[..., :64].contiguous())


@pytest.mark.parametrize("name,B,S,Hq,Hkv,causal", [
    ("config3a", 8, 4096, 32, 8, True),
    ("config3b", 2, 16384, 16, 16, False),
])
def test_full_size_configs_sampled(cuda_pkg, name, B, S, Hq, Hkv, causal):
    """Full-size configurations; the oracle recomputes a sample of (batch, head, row) triples."""
    g = torch.Generator(device="cuda").manual_seed(20260314)
    q = torch.randn((B, S, Hq, 128), device=DEV, dtype=torch.bfloat16, generator=g)
    k = torch.randn((B, S, Hkv, 128), device=DEV, dtype=torch.bfloat16, generator=g)
    v = torch.randn((B, S, Hkv, 128), device=DEV, dtype=torch.bfloat16, generator=g)
    out = cuda_pkg.flash_attn(q, k, v, causal=causal)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    pick = torch.Generator().manual_seed(3)
    groups = Hq // Hkv
    for _ in range(6):
        b = int(torch.randint(0, B, (1,), generator=pick))
        h = int(torch.randint(0, Hq, (1,), generator=pick))
        rows = torch.randint(0, S, (64,), generator=pick)
        rows[0], rows[1] = 0, S - 1
        qs = q[b, rows, h].cpu().float() / (128 ** 0.5)
        kf = k[b, :, h // groups].cpu().float()
        vf = v[b, :, h // groups].cpu().float()
        scores = qs @ kf.T
        if causal:
            scores = scores.masked_fill(torch.arange(S).unsqueeze(0) > rows.unsqueeze(1), float("-inf"))
        want = torch.softmax(scores, dim=-1) @ vf
        torch.testing.assert_close(out[b, rows, h].cpu().float(), want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("lengths,Hq,Hkv", [
    ([5, 300, 1, 128, 257], 8, 1),      # the reference's head layout, ragged lengths
    ([1000, 24, 640], 4, 2),
    ([128, 128], 2, 2),
])
@pytest.mark.parametrize("causal", [True, False])
def test_packed_variable_length(cuda_pkg, lengths, Hq, Hkv, causal):
    """flash_attn(q, k, v, seq_ptr, max_seq_len): every sequence equals the oracle run on it alone."""
    total = sum(lengths)
    g = torch.Generator().manual_seed(total + Hq)
    q = torch.randn((total, Hq, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((total, Hkv, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((total, Hkv, 128), generator=g).to(torch.bfloat16)
    seq_ptr = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=torch.int32)
    out = cuda_pkg.flash_attn_packed(q.to(DEV), k.to(DEV), v.to(DEV), seq_ptr.to(DEV), max(lengths), causal=causal)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    out = out.cpu()
    for i, n in enumerate(lengths):
        a = int(seq_ptr[i])
        want = attention_oracle.attention_reference(q[a:a + n].unsqueeze(0), k[a:a + n].unsqueeze(0),
                                                    v[a:a + n].unsqueeze(0), causal=causal)[0]
        torch.testing.assert_close(out[a:a + n].float(), want.float(), rtol=RTOL, atol=ATOL)


def test_packed_matches_batched_layout(cuda_pkg):
    """The harness layout [B,S,H,D] is the packed layout with seq_ptr = arange(B+1) * S
    (datasets/inference/attention/lumen/model.py:64-79 of the reference): identical bits."""
    q, k, v = attention_oracle.attention_inputs(3, 200, 8, 2, 128, 21)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = cuda_pkg.flash_attn(qd, kd, vd, causal=True)
    seq_ptr = (torch.arange(4, dtype=torch.int32) * 200).to(DEV)
    b = cuda_pkg.flash_attn_packed(qd.view(600, 8, 128), kd.view(600, 2, 128), vd.view(600, 2, 128), seq_ptr, 200)
    torch.cuda.synchronize()
    assert torch.equal(a.view(600, 8, 128), b)
    with pytest.raises(TypeError):
        cuda_pkg.flash_attn_packed(qd.view(600, 8, 128), kd.view(600, 2, 128), vd.view(600, 2, 128), [0, 600], 600)
    with pytest.raises(ValueError, match="longest sequence"):
        cuda_pkg.flash_attn_packed(qd.view(600, 8, 128), kd.view(600, 2, 128), vd.view(600, 2, 128), seq_ptr, 601)
