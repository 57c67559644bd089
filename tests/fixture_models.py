"""The small models behind the reference decode fixtures (tests/golden/decoder_*.npz,
moe_decode.npz), rebuilt from their seeds in the forms the oracles and the B200 decoders take.

Test support only: weights come from ``tests/golden/make_decoder_fixtures.py`` (numpy seeds),
so nothing here reads the reference."""
from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))

import make_decoder_fixtures as mdf  # noqa: E402

# A greedy token may differ from the reference's only where the reference's own top-1/top-2
# logit margin is below this bound (the bf16 contract's logit error measured on these models
# is under 0.012 against logits of magnitude 2.5-4.5).
NEAR_TIE = 0.02


def dense_oracle_weights() -> dict[str, np.ndarray]:
    """The dense model in the oracles' naming (``name.codes`` / ``name.scales`` + fp32)."""
    qrows, fp32 = mdf.dense_blocks()
    w: dict[str, np.ndarray] = {}
    for name, (codes, scales) in qrows.items():
        w[name + ".codes"], w[name + ".scales"] = codes, scales
    w.update(fp32)
    return w


def dense_config() -> dict:
    return dict(mdf.DENSE_CONFIG)


def moe_config() -> SimpleNamespace:
    c = mdf.MOE_CONFIG
    return SimpleNamespace(num_layers=c["num_hidden_layers"], hidden=c["hidden_size"], heads=c["num_attention_heads"],
                           kv_heads=c["num_key_value_heads"], head_dim=c["head_dim"], experts=c["num_experts"],
                           top_k=c["num_experts_per_tok"], expert_ffn=c["moe_intermediate_size"],
                           vocab=c["vocab_size"], rope_theta=c["rope_theta"], eps=c["rms_norm_eps"],
                           norm_topk=c["norm_topk_prob"])


def moe_host_weights() -> dict:
    """The MoE model as ``MoeWeights.to_host()`` lays it out: q/k/v stacked, expert pages packed
    (gate and up codes as one [2F, H] block) in the expert page layout."""
    import torch

    from mrun_b200.moe import ExpertPageLayout, pack_expert_page

    c = moe_config()
    m = mdf.moe_model()
    layout = ExpertPageLayout.create(c.hidden, c.expert_ffn)
    layers = []
    for L in m["layers"]:
        pages = torch.zeros(c.experts, layout.page_stride, dtype=torch.uint8)
        for e in range(c.experts):
            gu = np.concatenate([L["gate"][e][0], L["up"][e][0]])
            gus = np.concatenate([L["gate"][e][1], L["up"][e][1]])
            pack_expert_page(layout, torch.from_numpy(gu), torch.from_numpy(gus), torch.from_numpy(L["down"][e][0]),
                             torch.from_numpy(L["down"][e][1]), pages[e])
        qkv = (np.concatenate([L["q"][0], L["k"][0], L["v"][0]]), np.concatenate([L["q"][1], L["k"][1], L["v"][1]]))
        layers.append({"qkv": qkv, "o": L["o"], "router": L["router"], "q_norm": L["q_norm"], "k_norm": L["k_norm"],
                       "ln1": L["ln1"], "ln2": L["ln2"], "pages": pages.numpy()})
    return {"embed": m["embed"], "final_norm": m["final_norm"], "head": m["head"], "layout": layout.as_dict(),
            "layers": layers}


def moe_device_weights(device):
    """``MoeWeights`` on ``device`` holding exactly the fixture model."""
    import torch

    from mrun_b200.dense_engine import QRow
    from mrun_b200.moe import ExpertPageLayout
    from mrun_b200.moe_engine import MoeConfig, MoeLayer, MoeWeights

    c = moe_config()
    cfg = MoeConfig(num_layers=c.num_layers, hidden=c.hidden, heads=c.heads, kv_heads=c.kv_heads,
                    head_dim=c.head_dim, experts=c.experts, top_k=c.top_k, expert_ffn=c.expert_ffn, vocab=c.vocab,
                    rope_theta=c.rope_theta, eps=c.eps, norm_topk=c.norm_topk)
    host = moe_host_weights()

    def qrow(pair):
        return QRow(torch.from_numpy(pair[0].copy()).to(device), torch.from_numpy(pair[1].copy()).to(device))

    def vec(a, dtype):
        return torch.from_numpy(np.asarray(a, np.float32).copy()).to(device).to(dtype)

    layers = [MoeLayer(qkv=qrow(L["qkv"]), o=qrow(L["o"]), router=qrow(L["router"]),
                       q_norm=vec(L["q_norm"], torch.bfloat16), k_norm=vec(L["k_norm"], torch.bfloat16),
                       ln1=vec(L["ln1"], torch.float32), ln2=vec(L["ln2"], torch.float32),
                       pages=torch.from_numpy(L["pages"].copy()).to(device)) for L in host["layers"]]
    return MoeWeights(cfg=cfg, layout=ExpertPageLayout(**host["layout"]), embed=qrow(host["embed"]), layers=layers,
                      final_norm=vec(host["final_norm"], torch.float32), head=qrow(host["head"]), expert_first=0,
                      experts_local=c.experts)


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}
