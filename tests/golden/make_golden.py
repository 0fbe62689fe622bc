"""Generate the golden fixtures in this directory from the REFERENCE's own code.

Run where a checkout of the reference exists:

    python tests/golden/make_golden.py --reference /path/to/lumen-sosp26-ae

It imports, unmodified,
  * prompts/kernelbench/1_gemm.py            Model
  * prompts/kernelbench/2_attention.py       Model  (module globals set to the case's heads)
  * scripts/benchmark/backend_attn.py        _attention_reference, SharedInputs
  * scripts/benchmark/backend_moe.py         _moe_reference, SharedInputs
  * prompts/kernelbench/3_fused_moe.py       Model  (module global TOPK set)
  * datasets/inference/moe/lumen/model.py    _build_sorted_routes
runs them on small seeded CPU inputs, checks that the oracle/ restatement agrees with
them, and stores inputs + reference outputs as .npz (bf16 kept as raw uint16 bits).
The fixtures are what tests replay where the reference checkout does not exist.
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import attention_oracle, gemm_oracle, moe_oracle  # noqa: E402


def load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def max_ulp_bf16(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of haohui/lumen-sosp26-ae")
    ref = Path(ap.parse_args().reference)
    sys.path.insert(0, str(ref / "scripts" / "benchmark"))
    torch.manual_seed(0)

    # ------------------------------------------------------------------ GEMM
    gemm_mod = load(ref / "prompts/kernelbench/1_gemm.py", "ref_gemm_prompt")
    cases = {}
    for name, (m, n, k, seed, bstd) in {
        "small": (48, 40, 64, 20260312, 1.0),
        "ragged": (130, 72, 200, 20260313, 0.02),
    }.items():
        a, b = gemm_oracle.gemm_inputs(m, n, k, seed, bstd)
        ref_out = gemm_mod.Model()(a, b)  # torch.matmul(A, B.T) in bf16 on CPU
        ora = gemm_oracle.gemm_reference(a, b)
        # CPU bf16 matmul accumulates in fp32 and rounds once: identical up to 1 bf16 ulp
        torch.testing.assert_close(ora.float(), ref_out.float(), rtol=1e-2, atol=1e-2)
        cases[f"{name}_a"] = bits(a)
        cases[f"{name}_b"] = bits(b)
        cases[f"{name}_out"] = bits(ref_out)
    np.savez_compressed(HERE / "gemm.npz", **cases)

    # ------------------------------------------------------------- attention
    attn_prompt = load(ref / "prompts/kernelbench/2_attention.py", "ref_attn_prompt")
    backend_attn = load(ref / "scripts/benchmark/backend_attn.py", "ref_backend_attn")
    cases = {}
    for name, (B, S, Hq, Hkv, seed) in {
        "gqa": (1, 80, 4, 2, 20260314),
        "mqa": (2, 45, 8, 1, 20260315),
    }.items():
        q, k, v = attention_oracle.attention_inputs(B, S, Hq, Hkv, 128, seed)
        shared = backend_attn.SharedInputs(q_bshd=q, k_bshd=k, v_bshd=v)
        for causal in (True, False):
            ref_out = backend_attn._attention_reference(shared, causal=causal)
            ora = attention_oracle.attention_reference(q, k, v, causal=causal, q_chunk=32)
            torch.testing.assert_close(ora.float(), ref_out.float(), rtol=2e-2, atol=2e-2)
            cases[f"{name}_out_{'causal' if causal else 'full'}"] = bits(ref_out)
        # the KernelBench-style Model (causal only) pins the explicit-softmax form too
        attn_prompt.num_q_heads, attn_prompt.num_kv_heads = Hq, Hkv
        model_out = attn_prompt.Model()(q, k, v)
        ora = attention_oracle.attention_reference(
            q, k, v, causal=True, scale=attention_oracle.SM_SCALE_D128, q_chunk=32)
        torch.testing.assert_close(ora.float(), model_out.float(), rtol=1e-2, atol=1e-2)
        cases[f"{name}_out_model_causal"] = bits(model_out)
        cases[f"{name}_q"], cases[f"{name}_k"], cases[f"{name}_v"] = bits(q), bits(k), bits(v)
    np.savez_compressed(HERE / "attention.npz", **cases)

    # ------------------------------------------------------------------- MoE
    backend_moe = load(ref / "scripts/benchmark/backend_moe.py", "ref_backend_moe")
    lumen_moe = load(ref / "datasets/inference/moe/lumen/model.py", "ref_lumen_moe_model")
    moe_prompt = load(ref / "prompts/kernelbench/3_fused_moe.py", "ref_moe_prompt")
    cases = {}
    for name, (T, H, I, E, k, seed, with_router) in {
        "mixtral_like": (40, 128, 128, 8, 2, 20260319, True),
        "fine_grained": (33, 128, 128, 32, 8, 20260320, False),
    }.items():
        d = moe_oracle.moe_inputs(T, H, I, E, seed, with_router=with_router)
        logits = moe_oracle.router_logits(d["x"], d["w_router"]) if with_router else d["logits"]
        # reference routing: topk(sorted=True) + softmax(topk_val)  (backend_moe.py:131-139)
        tv, ti = torch.topk(logits, k=k, dim=-1, largest=True, sorted=True)
        ref_ids = ti.to(torch.int32).contiguous()
        ref_w = torch.softmax(tv, dim=-1).to(torch.float32).contiguous()
        ids, w = moe_oracle.route_topk(logits, k)
        assert torch.equal(ids, ref_ids), "oracle routing differs from torch.topk"
        torch.testing.assert_close(w, ref_w, rtol=0, atol=0)
        # reference permutation
        r_tok, r_w, r_eid, r_nv = lumen_moe._build_sorted_routes(
            topk_ids=ref_ids, topk_weights=ref_w, experts=E)
        o = moe_oracle.build_sorted_routes(ref_ids.numpy(), ref_w.numpy(), E)
        assert np.array_equal(o[0], r_tok.numpy()) and np.array_equal(o[1], r_w.numpy())
        assert np.array_equal(o[2], r_eid.numpy()) and np.array_equal(o[3], r_nv.numpy())
        # reference expert compute with unit scales (backend_moe.py:469-504)
        ones = lambda *s: torch.ones(s, dtype=torch.float32)  # noqa: E731
        shared = backend_moe.SharedInputs(
            input_q=d["x"], topk_weights=ref_w, topk_ids=ref_ids, input_scale=ones(T, H // 128))
        weights = {
            "w1_q": d["w13"], "w2_q": d["w2"],
            "fc1_scale": ones(E, (2 * I // 128) * (H // 128)),
            "fc2_scale": ones(E, (H // 128) * (I // 128)),
        }
        ref_out = backend_moe._moe_reference(inputs=shared, weights=weights, dim=H, inter_dim=I, experts=E)
        ora = moe_oracle.moe_reference(d["x"], d["w13"], d["w2"], ref_ids, ref_w)
        assert torch.equal(ora, ref_out), "oracle MoE differs from _moe_reference"
        # the all-experts einsum Model of the task prompt agrees within rounding
        moe_prompt.TOPK = k
        model_out = moe_prompt.Model()(d["x"], d["w13"], d["w2"], ref_w, ref_ids,
                                       shared.input_scale, weights["fc1_scale"], weights["fc2_scale"])
        torch.testing.assert_close(model_out.float(), ref_out.float(), rtol=2e-2, atol=2e-2)
        cases[f"{name}_x"] = bits(d["x"])
        cases[f"{name}_w13"] = bits(d["w13"])
        cases[f"{name}_w2"] = bits(d["w2"])
        if with_router:
            cases[f"{name}_w_router"] = bits(d["w_router"])
        cases[f"{name}_logits"] = logits.numpy()
        cases[f"{name}_topk_ids"] = ref_ids.numpy()
        cases[f"{name}_topk_weights"] = ref_w.numpy()
        cases[f"{name}_sorted_token_ids"] = r_tok.numpy()
        cases[f"{name}_sorted_weights"] = r_w.numpy()
        cases[f"{name}_sorted_expert_ids"] = r_eid.numpy()
        cases[f"{name}_num_valid_ids"] = r_nv.numpy()
        cases[f"{name}_out"] = bits(ref_out)
    # routing-only case at the fine-grained expert count, with empty experts and ragged loads
    g = torch.Generator().manual_seed(20260321)
    logits = torch.randn((300, 256), generator=g)
    tv, ti = torch.topk(logits, k=8, dim=-1, largest=True, sorted=True)
    ref_ids = ti.to(torch.int32).contiguous()
    ref_w = torch.softmax(tv, dim=-1).to(torch.float32).contiguous()
    # force some experts empty and one overloaded
    ref_ids[ref_ids >= 250] = 3
    r_tok, r_w, r_eid, r_nv = lumen_moe._build_sorted_routes(topk_ids=ref_ids, topk_weights=ref_w, experts=256)
    o = moe_oracle.build_sorted_routes(ref_ids.numpy(), ref_w.numpy(), 256)
    assert all(np.array_equal(a, b.numpy()) for a, b in zip(o[:4], (r_tok, r_w, r_eid, r_nv)))
    cases.update(routes_topk_ids=ref_ids.numpy(), routes_topk_weights=ref_w.numpy(),
                 routes_sorted_token_ids=r_tok.numpy(), routes_sorted_weights=r_w.numpy(),
                 routes_sorted_expert_ids=r_eid.numpy(), routes_num_valid_ids=r_nv.numpy())
    np.savez_compressed(HERE / "moe.npz", **cases)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
