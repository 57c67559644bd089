"""Generate golden vectors by running the mrun reference itself on seeded inputs.

Run where the reference source is importable (it is not shipped with this repository):

    PYTHONPATH=<mrun checkout>/src python tests/golden/make_golden.py

Every fixture records the reference function (file:line) that produced it. The committed
``.npz`` files are what the tests read; nothing at test time imports the reference.
Inputs are seeded (torch.manual_seed / numpy default_rng) so they are reproducible.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype is torch.bfloat16:
        return t.float().numpy()
    return t.detach().cpu().numpy()


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def qrow_fixtures() -> None:
    from mrun.engine.kernels.dense_qstore_cuda import (  # noqa: PLC0415
        CompactQRowPage,
        dequantized_reference_matmul,
        fused_qrow_swiglu_reference,
        fused_residual_rms_norm_reference,
        qrow_top2_reference,
        rerank_qrow_candidates_fp32,
        stable_rms_norm_reference,
    )
    from mrun.engine.kernels.qstore import _dequant_qrow  # noqa: PLC0415
    from mrun.engine.kernels.qstore_build import _quant_row_int8  # noqa: PLC0415

    out: dict[str, np.ndarray] = {}
    # quantiser: N(0, 0.02) rows, one all-zero row, one row with exact half-step ties
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((48, 160)) * 0.02).astype(np.float32)
    w[5] = 0.0
    w[7] = np.linspace(-1.0, 1.0, 160, dtype=np.float32)
    w[7, :4] = np.float32(127.0 / 254.0) * np.array([1, 3, -5, 7], np.float32) / np.float32(127.0)
    q, s = _quant_row_int8(w)
    out.update(quant_w=w, quant_q=q, quant_s=s)

    # QStore.matmul fp32 semantics (engine/kernels/qstore.py:1082-1092)
    torch.manual_seed(1)
    x32 = torch.randn(6, 160)
    W = torch.from_numpy(_dequant_qrow(q, s).numpy())
    out["mm32_x"] = _np(x32)
    out["mm32_y"] = _np(x32 @ W.T)

    # W8A16 contract (engine/kernels/dense_qstore_cuda.py:1003-1013)
    torch.manual_seed(2)
    page_w = (torch.randn(96, 256) * 0.02).numpy().astype(np.float32)
    pq, ps = _quant_row_int8(page_w)
    page = CompactQRowPage("p", 0, 96, 256, torch.from_numpy(pq.copy()), torch.from_numpy(ps.copy()))
    xb = torch.randn(5, 256).to(torch.bfloat16)
    out.update(w16_q=pq, w16_s=ps, w16_x=_np(xb), w16_y=_np(dequantized_reference_matmul(page, xb)))

    # paired SwiGLU (engine/kernels/dense_qstore_cuda.py:1037-1049)
    torch.manual_seed(3)
    gq, gs = _quant_row_int8((torch.randn(64, 128) * 0.05).numpy())
    uq, us = _quant_row_int8((torch.randn(64, 128) * 0.05).numpy())
    gpage = CompactQRowPage("g", 0, 64, 128, torch.from_numpy(gq.copy()), torch.from_numpy(gs.copy()))
    upage = CompactQRowPage("u", 0, 64, 128, torch.from_numpy(uq.copy()), torch.from_numpy(us.copy()))
    xs = (torch.randn(3, 128) * 2).to(torch.bfloat16)
    out.update(sw_gq=gq, sw_gs=gs, sw_uq=uq, sw_us=us, sw_x=_np(xs),
               sw_y=_np(fused_qrow_swiglu_reference(gpage, upage, xs)))

    # residual RMSNorm (engine/kernels/dense_qstore_cuda.py:1390-1408)
    torch.manual_seed(4)
    res = torch.randn(4, 512).to(torch.bfloat16)
    upd = torch.randn(4, 512).to(torch.bfloat16)
    nw = torch.rand(512) + 0.5
    r, n = fused_residual_rms_norm_reference(res, upd, nw, 1e-6)
    out.update(rr_res=_np(res), rr_upd=_np(upd), rr_w=_np(nw), rr_r=_np(r), rr_n=_np(n))

    # RMSNorm (engine/kernels/dense_qstore_cuda.py:1462-1470)
    rn_x = torch.randn(3, 512).to(torch.bfloat16)
    out.update(rn_x=_np(rn_x), rn_y=_np(stable_rms_norm_reference(rn_x, nw, 1e-6)))

    # top-2 head + fp32 rerank (engine/kernels/dense_qstore_cuda.py:1155-1235)
    torch.manual_seed(5)
    hq, hs = _quant_row_int8((torch.randn(300, 64) * 0.02).numpy())
    hpage = CompactQRowPage("lm_head", 0, 300, 64, torch.from_numpy(hq.copy()), torch.from_numpy(hs.copy()))
    hx = torch.randn(4, 64).to(torch.bfloat16)
    idx, val = qrow_top2_reference(hpage, hx, semantic_row_count=290)
    best, best_val = rerank_qrow_candidates_fp32(hpage, hx, idx)
    out.update(hd_q=hq, hd_s=hs, hd_x=_np(hx), hd_top2=_np(idx), hd_best=_np(best), hd_best_val=_np(best_val))
    np.savez_compressed(HERE / "qrow.npz", **out)


def config1_fixture() -> None:
    """The 8 x 2048 x 2048 W8A16 / W8A8 linear at full size, recorded as checksums plus the fp32 outputs."""
    from mrun.engine.kernels.qstore import _dequant_qrow  # noqa: PLC0415
    from mrun.engine.kernels.qstore_build import _quant_row_int8  # noqa: PLC0415
    from mrun.engine.kernels.w8a8 import _int8_gemm, w8a8_matmul  # noqa: PLC0415

    torch.manual_seed(0)
    x = torch.randn(8, 2048)
    w = torch.randn(2048, 2048) * 0.02
    q, s = _quant_row_int8(w.numpy())
    y16 = x @ _dequant_qrow(q, s).T
    qt, st = torch.from_numpy(q.copy()), torch.from_numpy(s.copy())
    y8 = w8a8_matmul(qt, st, x, protect_k=0)
    # the int32 accumulator of the W8A8 path (engine/kernels/w8a8.py:117-124)
    act_scale = x.abs().amax(dim=1, keepdim=True) / 127.0
    act_scale = torch.where(act_scale == 0, torch.ones_like(act_scale), act_scale)
    qx = torch.round(x / act_scale).clamp_(-127, 127).to(torch.int8)
    acc = _int8_gemm(qx, qt, True)
    np.savez_compressed(
        HERE / "config1.npz",
        codes_sha=np.array(sha(q)),
        scales_sha=np.array(sha(s)),
        y_w8a16=y16.numpy(),
        y_w8a8=y8.numpy(),
        qx=qx.numpy(),
        act_scale=act_scale.numpy(),
        acc_sha=np.array(sha(acc.numpy())),
        acc_rows0=acc[:2].numpy(),
    )


def w8a8_fixtures() -> None:
    from mrun.engine.kernels.w8a8 import _int8_gemm, w8a8_matmul  # noqa: PLC0415

    # the reference's own test setup (tests/test_w8a8.py:14-22)
    torch.manual_seed(0)
    q_w = torch.randint(-127, 128, (64, 128), dtype=torch.int8)
    sc_w = torch.rand(64) * 0.02 + 1e-3
    x = torch.randn(5, 128)
    x[:, torch.randperm(128)[:3]] *= 300.0
    out = {
        "q_w": q_w.numpy(),
        "sc_w": sc_w.numpy(),
        "x": x.numpy(),
        "y_k0": w8a8_matmul(q_w, sc_w, x, protect_k=0).numpy(),
        "y_k4": w8a8_matmul(q_w, sc_w, x, protect_k=4).numpy(),
    }
    q_x = torch.randint(-127, 128, (7, 128), dtype=torch.int8)
    out["gemm_qx"] = q_x.numpy()
    out["gemm_acc"] = _int8_gemm(q_x, q_w, False).numpy()
    np.savez_compressed(HERE / "w8a8.npz", **out)


def attention_fixtures() -> None:
    from mrun.engine.kernels.dense_qstore_cuda import segmented_decode_attention_reference  # noqa: PLC0415
    from mrun.engine.kernels.segmented_gqa_decode import segmented_gqa_decode_reference  # noqa: PLC0415

    torch.manual_seed(6)
    q = torch.randn(2, 1, 8, 64).to(torch.bfloat16)
    ck = torch.randn(2, 40, 2, 64).to(torch.bfloat16)
    cv = torch.randn(2, 40, 2, 64).to(torch.bfloat16)
    kn = torch.randn(2, 1, 2, 64).to(torch.bfloat16)
    vn = torch.randn(2, 1, 2, 64).to(torch.bfloat16)
    lengths = torch.tensor([17, 33])
    seg = segmented_decode_attention_reference(q, ck, cv, kn, vn, lengths)

    gq = torch.randn(3, 8, 64).to(torch.bfloat16)
    kc = torch.randn(4, 2, 48, 64).to(torch.bfloat16)
    vc = torch.randn(4, 2, 48, 64).to(torch.bfloat16)
    slots = torch.tensor([2, 0, 3])
    lens = torch.tensor([5, 48, 31])
    gqa = segmented_gqa_decode_reference(gq, kc, vc, slots, lens)
    np.savez_compressed(
        HERE / "attention.npz",
        seg_q=_np(q), seg_ck=_np(ck), seg_cv=_np(cv), seg_kn=_np(kn), seg_vn=_np(vn),
        seg_len=lengths.numpy(), seg_out=_np(seg),
        gqa_q=_np(gq), gqa_kc=_np(kc), gqa_vc=_np(vc), gqa_slots=slots.numpy(),
        gqa_len=lens.numpy(), gqa_out=_np(gqa),
    )


def moe_fixtures() -> None:
    from mrun.engine.olmoe_cuda import grouped_route_tensors_with_inverse  # noqa: PLC0415
    from mrun.engine.qwen3_moe_cuda import stable_route_reduce  # noqa: PLC0415

    out = {}
    # router maths (engine/qwen3_moe_cuda.py:3700-3707): softmax(fp32) -> topk -> renorm -> bf16
    torch.manual_seed(7)
    logits = torch.randn(32, 128)
    probs = torch.softmax(logits.float(), dim=-1)
    tw, ti = probs.topk(8, dim=-1)
    tw = (tw / tw.sum(-1, keepdim=True)).to(torch.bfloat16)
    out.update(router_logits=logits.numpy(), router_idx=ti.numpy(), router_w=_np(tw))

    # route compiler, CPU branch (engine/olmoe_cuda.py:1064-1089)
    tok, coef, starts, counts, inv, _ = grouped_route_tensors_with_inverse(ti, tw.float(), num_experts=128)
    out.update(route_tok=tok.numpy(), route_coef=coef.numpy(), route_starts=starts.numpy(),
               route_counts=counts.numpy(), route_inv=inv.numpy())

    # stable reduce, CPU branch (engine/qwen3_moe_cuda.py:2654-2664)
    eo = torch.randn(32 * 8, 96).to(torch.bfloat16)
    selected = torch.arange(128)
    red = stable_route_reduce(eo, coef, tok, counts, ti, selected, inverse_assignments=inv)
    out.update(reduce_eo=_np(eo), reduce_out=red.numpy())
    np.savez_compressed(HERE / "moe.npz", **out)


def main() -> int:
    try:
        import mrun  # noqa: F401, PLC0415
    except ImportError:
        print("the mrun reference is not importable; set PYTHONPATH to its src/ directory", file=sys.stderr)
        return 2
    torch.set_num_threads(max(1, torch.get_num_threads()))
    qrow_fixtures()
    config1_fixture()
    w8a8_fixtures()
    attention_fixtures()
    moe_fixtures()
    for path in sorted(HERE.glob("*.npz")):
        print(path.name, path.stat().st_size)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
