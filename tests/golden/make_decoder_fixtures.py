"""Greedy-decode fixtures from the reference's own decoders (run where the reference sources
are; the outputs are committed, so tests need no reference at run time).

The models are small and fully determined by a seed: ``build_dense_store`` writes a dense
Qwen2-style int8 QStore and ``moe_model`` draws a Qwen3-MoE-style int8 model, both from
``numpy.random.default_rng``; tests rebuild the same weights from the same seeds instead of
reading committed weight files. For each model the fixture records the prompt, every greedy
token, and per step the top-1 / top-2 logits and their margin, so a test can tell a genuine
near-tie from a wrong token.

* ``decoder_fp32.npz`` -- ``paged_forward_kv`` (engine/kernels/paged_forward.py:1016-1107), the
  reference's CPU fp32 decode, over the dense store (legacy schema): prefill, then 256 steps.
* ``decoder_bf16.npz`` -- ``DenseQStoreTarget`` (engine/dense_qstore_cuda.py:506-1290) on the
  CPU with the eager kernels (``require_triton=False``): the dense CUDA engine's bf16 contract
  (bf16 weights per projection, bf16 activation boundaries, fp32 exact head), same prompt
  and 256 steps.
* ``moe_decode.npz`` -- ``Qwen3MoeDecodeRuntime.forward`` (engine/qwen3_moe_cuda.py:3536) on
  the CPU in fp32 with an injected CPU int8 expert backend (the runtime takes any ``.moe``
  object, as the reference's tests do, tests/test_qwen3_moe_cuda.py:1305-1334): prefill of
  each prompt, then 64 steps. The backend computes each routed expert as
  ``silu(x W_g^T) * (x W_u^T)`` then ``W_d``, with ``W = codes * scale`` in fp32, and adds the
  k outputs weighted by the router weights in rank order (engine/qwen3_moe_cuda.py:2740-2761,
  2654-2664); the reference has no CPU expert GEMM of its own.

Usage: ``python tests/golden/make_decoder_fixtures.py <reference src directory>``.
"""
from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

DENSE_CONFIG = {
    "num_hidden_layers": 4, "hidden_size": 512, "num_attention_heads": 8, "num_key_value_heads": 2,
    "head_dim": 128, "intermediate_size": 1024, "vocab_size": 4096, "rope_theta": 1e6, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 4096, "tie_word_embeddings": False,
}
DENSE_SEED, DENSE_PROMPT, DENSE_STEPS = 20261202, 32, 256

MOE_CONFIG = {
    "num_hidden_layers": 2, "hidden_size": 256, "num_attention_heads": 4, "num_key_value_heads": 2,
    "head_dim": 128, "num_experts": 16, "num_experts_per_tok": 4, "moe_intermediate_size": 128,
    "vocab_size": 1024, "rope_theta": 1e6, "rms_norm_eps": 1e-6, "norm_topk_prob": True,
}
MOE_SEED, MOE_PROMPTS, MOE_STEPS = 7, (12, 20), 64


def _quant(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference quantiser (engine/kernels/qstore_build.py:496-501), via the oracle."""
    sys.path.insert(0, str(REPO))
    from oracle.qrow import quant_row_int8

    return quant_row_int8(w.astype(np.float32))


def dense_blocks(seed: int = DENSE_SEED) -> tuple[dict, dict]:
    """qrow and fp32 blocks (canonical names) of the dense fixture model."""
    c = DENSE_CONFIG
    rng = np.random.default_rng(seed)
    h, hd, f, v = c["hidden_size"], c["head_dim"], c["intermediate_size"], c["vocab_size"]
    qd, kd = c["num_attention_heads"] * hd, c["num_key_value_heads"] * hd

    def mat(rows, cols, std=0.02):
        return _quant(rng.standard_normal((rows, cols)).astype(np.float32) * std)

    qrows = {"embed": mat(v, h, 1.0)}
    fp32 = {}
    for i in range(c["num_hidden_layers"]):
        qrows[f"L{i}.q"] = mat(qd, h)
        qrows[f"L{i}.k"] = mat(kd, h)
        qrows[f"L{i}.v"] = mat(kd, h)
        qrows[f"L{i}.o"] = mat(h, qd)
        qrows[f"L{i}.gate"] = mat(f, h)
        qrows[f"L{i}.up"] = mat(f, h)
        qrows[f"L{i}.down"] = mat(h, f)
        for name, n in (("q.bias", qd), ("k.bias", kd), ("v.bias", kd)):
            fp32[f"L{i}.{name}"] = (rng.standard_normal(n) * 0.02).astype(np.float32)
        fp32[f"L{i}.ln1"] = (1.0 + 0.05 * rng.standard_normal(h)).astype(np.float32)
        fp32[f"L{i}.ln2"] = (1.0 + 0.05 * rng.standard_normal(h)).astype(np.float32)
    fp32["norm.final"] = (1.0 + 0.05 * rng.standard_normal(h)).astype(np.float32)
    qrows["lm_head"] = mat(v, h, 0.05)
    return qrows, fp32


def dense_prompt() -> np.ndarray:
    return np.random.default_rng(DENSE_SEED + 1).integers(0, DENSE_CONFIG["vocab_size"], DENSE_PROMPT).astype(np.int64)


def build_dense_store(directory: Path, *, legacy: bool = False) -> dict:
    """Write the dense fixture model as an int8 QStore; ``legacy`` marks the manifest with the
    pre-v3 schema the reference opens without provenance digests."""
    sys.path.insert(0, str(REPO))
    from mrun_b200.qstore_build import write_qstore

    qrows, fp32 = dense_blocks()
    manifest = write_qstore(directory, qrows=qrows, fp32=fp32, config=dict(DENSE_CONFIG), arch="qwen2",
                            model_name=Path(directory).name)
    if legacy:
        manifest["schema_version"] = "mrun-qstore-int8-v2"
        (Path(directory) / "manifest.json").write_text(json.dumps(manifest))
    return manifest


def moe_model(seed: int = MOE_SEED) -> dict:
    """The MoE fixture model: int8 codes + fp32 scales for every matrix (dense projections,
    router, experts), norm weights, embedding and head."""
    c = MOE_CONFIG
    rng = np.random.default_rng(seed)
    h, hd, e, f, v = c["hidden_size"], c["head_dim"], c["num_experts"], c["moe_intermediate_size"], c["vocab_size"]
    qd, kd = c["num_attention_heads"] * hd, c["num_key_value_heads"] * hd

    def mat(rows, cols, std=0.02):
        return _quant(rng.standard_normal((rows, cols)).astype(np.float32) * std)

    def norm(n):  # bf16-representable, as the norm weights of a bf16 checkpoint are
        import torch

        w = torch.from_numpy((1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32))
        return w.to(torch.bfloat16).float().numpy()

    model = {"embed": mat(v, h, 1.0), "layers": []}
    for _ in range(c["num_hidden_layers"]):
        layer = {"q": mat(qd, h), "k": mat(kd, h), "v": mat(kd, h), "o": mat(h, qd), "router": mat(e, h, 0.05),
                 "ln1": norm(h), "ln2": norm(h), "q_norm": norm(hd), "k_norm": norm(hd),
                 "gate": [mat(f, h) for _ in range(e)], "up": [mat(f, h) for _ in range(e)],
                 "down": [mat(h, f) for _ in range(e)]}
        model["layers"].append(layer)
    model["final_norm"] = norm(h)
    model["head"] = mat(v, h, 0.05)
    return model


def moe_prompts() -> list[np.ndarray]:
    rng = np.random.default_rng(MOE_SEED + 1)
    return [rng.integers(0, MOE_CONFIG["vocab_size"], n).astype(np.int64) for n in MOE_PROMPTS]


def _top2(logits: np.ndarray) -> tuple[int, float, float]:
    order = np.argsort(-logits, kind="stable")
    return int(order[0]), float(logits[order[0]]), float(logits[order[1]])


def _record(tokens, top1, top2) -> dict:
    t1, t2 = np.asarray(top1, np.float32), np.asarray(top2, np.float32)
    return {"tokens": np.asarray(tokens, np.int64), "top1": t1, "top2": t2, "margin": t1 - t2}


def run_paged_forward(ref_root: Path, store_dir: Path) -> dict:
    import torch
    from mrun.engine.kernels.paged_forward import PagedKVCache, paged_forward_kv
    from mrun.engine.kernels.qstore import QStore

    torch.set_num_threads(os.cpu_count() or 1)
    store = QStore(store_dir.name, root=store_dir.parent, explicit_device="cpu", enable_prefetch_ring=False)
    c = DENSE_CONFIG
    cache = PagedKVCache(c["num_hidden_layers"], c["num_key_value_heads"], c["head_dim"],
                         DENSE_PROMPT + DENSE_STEPS + 1, "cpu")
    ids = dense_prompt()
    tokens, top1, top2 = [], [], []
    logits = paged_forward_kv(store, ids, cache).numpy()
    for _ in range(DENSE_STEPS + 1):
        tok, a, b = _top2(logits)
        tokens.append(tok)
        top1.append(a)
        top2.append(b)
        if len(tokens) > DENSE_STEPS:
            break
        logits = paged_forward_kv(store, np.array([tok], np.int64), cache).numpy()
    store.close()
    return {"prompt": ids, **_record(tokens, top1, top2)}


def run_dense_target(ref_root: Path, store_dir: Path) -> dict:
    import torch
    from mrun.engine.dense_qstore_cuda import DenseQStoreTarget
    from mrun.engine.kernels.dense_qstore_cuda import DenseQStore

    store = DenseQStore(store_dir.name, root=store_dir.parent, device="cpu", compute_dtype="bf16",
                        require_triton=False)
    target = DenseQStoreTarget(store, max_seq_len=DENSE_PROMPT + DENSE_STEPS + 1)
    cache = target.empty_cache(1)
    ids = torch.from_numpy(dense_prompt())[None, :]
    tokens, top1, top2 = [], [], []
    res = target.forward(ids, cache, return_logits=True)
    cache.commit(res.delta, [DENSE_PROMPT])
    while True:
        logits = res.logits[0, -1].float().numpy()
        tok = int(res.top1[0, -1])
        ref_tok, a, b = _top2(logits)
        assert ref_tok == tok, (ref_tok, tok)
        tokens.append(tok)
        top1.append(a)
        top2.append(b)
        if len(tokens) > DENSE_STEPS:
            break
        res = target.forward(torch.tensor([[tok]]), cache, return_logits=True)
        cache.commit(res.delta, [1])
    return {"prompt": ids[0].numpy(), **_record(tokens, top1, top2)}


class CpuInt8Experts:
    """A CPU int8 `.moe` backend for the reference runtime (fp32 arithmetic)."""

    def __init__(self, model: dict) -> None:
        import torch

        def deq(q):
            return torch.from_numpy(q[0].astype(np.float32) * q[1][:, None])

        self.gate = [[deq(q) for q in L["gate"]] for L in model["layers"]]
        self.up = [[deq(q) for q in L["up"]] for L in model["layers"]]
        self.down = [[deq(q) for q in L["down"]] for L in model["layers"]]

    def moe(self, layer, source, top_indices, top_weights, *, prefill=False):
        import torch

        x = source.float()
        out = torch.zeros_like(x)
        for t in range(x.shape[0]):
            acc = torch.zeros(x.shape[1])
            for r in range(top_indices.shape[1]):
                e = int(top_indices[t, r])
                g = x[t] @ self.gate[layer][e].T
                u = x[t] @ self.up[layer][e].T
                y = (torch.nn.functional.silu(g) * u) @ self.down[layer][e].T
                acc = acc + y * float(top_weights[t, r])
            out[t] = acc
        return out.to(source.dtype)


def run_moe_runtime(ref_root: Path) -> dict:
    import torch
    from mrun.engine.qwen3_moe_cuda import LayerWeights, Qwen3MoeDecodeRuntime
    from types import SimpleNamespace

    model = moe_model()
    c = MOE_CONFIG

    def deq(q):
        return torch.from_numpy(q[0].astype(np.float32) * q[1][:, None])

    layers = [LayerWeights(input_norm=torch.from_numpy(L["ln1"]), post_norm=torch.from_numpy(L["ln2"]),
                           q_norm=torch.from_numpy(L["q_norm"]), k_norm=torch.from_numpy(L["k_norm"]),
                           q_proj=deq(L["q"]), k_proj=deq(L["k"]), v_proj=deq(L["v"]), o_proj=deq(L["o"]),
                           router=deq(L["router"])) for L in model["layers"]]
    skeleton = SimpleNamespace(
        cfg={"num_hidden_layers": c["num_hidden_layers"], "num_attention_heads": c["num_attention_heads"],
             "num_key_value_heads": c["num_key_value_heads"], "head_dim": c["head_dim"],
             "hidden_size": c["hidden_size"], "num_experts_per_tok": c["num_experts_per_tok"],
             "rms_norm_eps": c["rms_norm_eps"], "rope_theta": c["rope_theta"], "norm_topk_prob": c["norm_topk_prob"]},
        device="cpu", dtype=torch.float32, embedding=deq(model["embed"]), layers=layers,
        final_norm=torch.from_numpy(model["final_norm"]), lm_head=deq(model["head"]))
    runtime = Qwen3MoeDecodeRuntime(skeleton, CpuInt8Experts(model))
    out = {}
    for p, prompt in enumerate(moe_prompts()):
        cache = runtime.new_cache(batch_size=1, capacity=len(prompt) + MOE_STEPS + 1)
        res = runtime.forward(torch.from_numpy(prompt)[None, :], cache=cache, capture_routes=True)
        tokens, top1, top2, routes = [], [], [], []
        while True:
            tok, a, b = _top2(res.logits[0].float().numpy())
            tokens.append(tok)
            top1.append(a)
            top2.append(b)
            if len(tokens) > MOE_STEPS:
                break
            res = runtime.forward(torch.tensor([[tok]]), cache=cache, capture_routes=True)
            if getattr(res, "routes", None) is not None:
                routes.append(np.stack([np.asarray(r.reshape(-1, r.shape[-1])[-1]) for r in res.routes]))
        rec = _record(tokens, top1, top2)
        out.update({f"p{p}_prompt": prompt, **{f"p{p}_{k}": v for k, v in rec.items()}})
        if routes:
            out[f"p{p}_routes"] = np.stack(routes).astype(np.int64)
    return out


def main() -> None:
    ref_src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MRUN_REFERENCE_SRC")
    if not ref_src:
        raise SystemExit("usage: make_decoder_fixtures.py <reference src directory>")
    sys.path.insert(0, ref_src)
    with tempfile.TemporaryDirectory() as tmp:
        store_dir = Path(tmp) / "dense_small"
        build_dense_store(store_dir, legacy=True)
        fp32 = run_paged_forward(Path(ref_src), store_dir)
        np.savez_compressed(HERE / "decoder_fp32.npz", **fp32)
        bf16 = run_dense_target(Path(ref_src), store_dir)
        np.savez_compressed(HERE / "decoder_bf16.npz", **bf16)
        shutil.rmtree(store_dir)
    moe = run_moe_runtime(Path(ref_src))
    np.savez_compressed(HERE / "moe_decode.npz", **moe)
    agree = int(np.sum(fp32["tokens"] == bf16["tokens"]))
    print(f"dense: {len(fp32['tokens'])} tokens, fp32/bf16 agree on {agree}; "
          f"min margin fp32 {fp32['margin'].min():.4f} bf16 {bf16['margin'].min():.4f}; moe arrays {len(moe)}")


if __name__ == "__main__":
    main()
