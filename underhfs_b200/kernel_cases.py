"""Single-kernel workloads for profiling and micro-benchmarking.

    python -m underhfs_b200.kernel_cases <case> [--iters N] [--time]
    UNDERHFS_ATTN_TRACE=1 python -m underhfs_b200._native_build && python -m underhfs_b200.kernel_cases {attn_fwd,attn_bwd} --trace

Each case builds its inputs once, launches one native kernel (or one fused
op) ``--iters`` times and checks the device status word.  Sizes are chosen
so the operands are larger than the 126 MB L2 where the kernel is
memory-bound, while the whole case stays at a few GB of device memory, which
keeps an ``ncu --set full`` capture of one launch short.  ``--time`` prints
the CUDA-event time per launch after three warm-up launches.  ``--trace``
(attn_fwd / attn_bwd) prints the per-block clock stamps of the attention
kernel for a few CTAs of the first head (SM cycles from the CTA's start).

Shapes follow the 125M TransformerLM step (16 x 1024 tokens, d_model 768,
12 heads of 64, MLP 3072, vocab 32000) unless the case says otherwise.
"""

from __future__ import annotations

import argparse
import sys
from typing import Callable

import torch

from underhfs_b200.ops import kernels as K

TOKENS = 16 * 1024


def _bf(*shape: int, scale: float = 1.0) -> torch.Tensor:
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def _case_gemm_fwd():
    x, w = _bf(TOKENS, 768), _bf(2304, 768, scale=0.03)
    return lambda: K.linear_fwd(x, w), 2.0 * TOKENS * 2304 * 768, 0


def _case_gemm_fwd_gelu():
    x, w, b = _bf(TOKENS, 768), _bf(3072, 768, scale=0.03), _bf(3072)
    return lambda: K.linear_fwd_gelu(x, w, b), 2.0 * TOKENS * 3072 * 768, 0


def _resid_case(n_out: int, n_in: int):
    """Linear with bias and the residual add fused in the epilogue (the
    out-projection is 768 x 768, fc2 768 x 3072)."""
    def case():
        x, w, b, r = _bf(TOKENS, n_in), _bf(n_out, n_in, scale=0.03), _bf(n_out), _bf(TOKENS, n_out)
        out = torch.empty(TOKENS, n_out, dtype=torch.bfloat16, device="cuda")
        return lambda: K.linear_fwd_resid(x, w, b, r, out=out), 2.0 * TOKENS * n_out * n_in, 0
    return case


def _resid_variant(block_n: int, cta_pair: int):
    """The out-projection (768 x 768, K 768) residual GEMM with a forced tile
    shape: block_n 128 or 256 on one SM, or the CTA pair."""
    def case():
        x, w, b, r = _bf(TOKENS, 768), _bf(768, 768, scale=0.03), _bf(768), _bf(TOKENS, 768)
        out = torch.empty(TOKENS, 768, dtype=torch.bfloat16, device="cuda")
        return (lambda: K.gemm_raw(TOKENS, 768, 768, x, 768, False, w, 768, False, out, 768, K.EPI_RESID, bias=b,
                                   aux=r, ld_aux=768, block_n=block_n, cta_pair=cta_pair),
                2.0 * TOKENS * 768 * 768, 0)
    return case


def _plain_case(n_out: int, n_in: int, pair: int):
    """Linear without bias or epilogue operand, for comparison with the
    residual variant of the same shape."""
    def case():
        x, w = _bf(TOKENS, n_in), _bf(n_out, n_in, scale=0.03)
        out = torch.empty(TOKENS, n_out, dtype=torch.bfloat16, device="cuda")
        return (lambda: K.gemm_raw(TOKENS, n_out, n_in, x, n_in, False, w, n_in, False, out, n_out, K.EPI_BF16,
                                   cta_pair=pair), 2.0 * TOKENS * n_out * n_in, 0)
    return case


def _wgrad_split_case(n_out: int, n_in: int, splits: int):
    def case():
        dy, x = _bf(TOKENS, n_out), _bf(TOKENS, n_in)
        dw = torch.zeros(n_out, n_in, device="cuda")
        return lambda: K.linear_wgrad_accum(dy, x, dw, splits=splits), 2.0 * TOKENS * n_out * n_in, 0
    return case


def _case_gemm_dgrad_dgelu():
    dy, w, u = _bf(TOKENS, 768), _bf(768, 3072, scale=0.03), _bf(TOKENS, 3072)
    return lambda: K.linear_dgrad(dy, w, gelu_in=u), 2.0 * TOKENS * 3072 * 768, 0


def _case_gemm_wgrad():
    dy, x = _bf(TOKENS, 2304), _bf(TOKENS, 768)
    dw = torch.zeros(2304, 768, device="cuda")
    return lambda: K.linear_wgrad_accum(dy, x, dw), 2.0 * TOKENS * 2304 * 768, 0


def _wgrad_case(n_out: int, n_in: int):
    def case():
        dy, x = _bf(TOKENS, n_out), _bf(TOKENS, n_in)
        dw = torch.zeros(n_out, n_in, device="cuda")
        return lambda: K.linear_wgrad_accum(dy, x, dw), 2.0 * TOKENS * n_out * n_in, 0
    return case


def _case_gemm_8192():
    a, b = _bf(8192, 8192, scale=0.02), _bf(8192, 8192, scale=0.02)
    return lambda: K.linear_fwd(a, b), 2.0 * 8192 ** 3, 0


def _attn_inputs(B=4, T=1024, H=12, D=64):
    qkv = _bf(B * T, 3 * H * D)
    o, lse = K.flash_attn_qkv(qkv, B, T, H, D, True)
    return qkv, o, lse, (B, T, H, D)


def _case_attn_fwd():
    qkv, _, _, (B, T, H, D) = _attn_inputs()
    return lambda: K.flash_attn_qkv(qkv, B, T, H, D, True), 2.0 * B * H * T * T * D, 0


def _case_attn_fwd16():
    """The forward at the 125M step's shape: B=16 T=1024 H=12 D=64, causal."""
    qkv, _, _, (B, T, H, D) = _attn_inputs(B=16)
    return lambda: K.flash_attn_qkv(qkv, B, T, H, D, True), 2.0 * B * H * T * T * D, 0


def _case_attn_bwd16():
    qkv, o, lse, (B, T, H, D) = _attn_inputs(B=16)
    do = _bf(B * T, H * D)
    return (lambda: K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True), 5.0 * B * H * T * T * D, 0)


def _case_attn_bwd():
    qkv, o, lse, (B, T, H, D) = _attn_inputs()
    do = _bf(B * T, H * D)
    return (lambda: K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True), 5.0 * B * H * T * T * D, 0)


def _case_rmsnorm_fwd():
    x, w = _bf(4 * TOKENS, 768), _bf(768)
    return lambda: K.rmsnorm(x, w, 1e-8), 0, 2 * x.numel() * 2


def _case_rmsnorm_bwd():
    x, w, dy = _bf(4 * TOKENS, 768), _bf(768), _bf(4 * TOKENS, 768)
    _, rstd = K.rmsnorm(x, w, 1e-8)
    dres = _bf(4 * TOKENS, 768)
    dw = torch.zeros(768, device="cuda")
    return lambda: K.rmsnorm_backward(dy, x, w, rstd, dres=dres, dw32=dw), 0, 4 * x.numel() * 2


def _case_softmax_ce():
    rows, cols = 4096, 32000
    logits = _bf(rows, cols)
    tg = torch.randint(0, cols, (rows,), device="cuda", dtype=torch.int64)
    dl = torch.empty_like(logits)
    return lambda: K.softmax_cross_entropy(logits, tg, dl, 1.0 / rows), 0, 2 * logits.numel() * 2


def _case_embedding_fwd():
    tok, pos = _bf(32000, 768), _bf(1024, 768)
    ids = torch.randint(0, 32000, (4 * TOKENS,), device="cuda", dtype=torch.int64)
    return lambda: K.embedding(ids, tok, pos, 1024), 0, 2 * ids.numel() * 768 * 2


def _case_embedding_bwd():
    ids = torch.randint(0, 32000, (4 * TOKENS,), device="cuda", dtype=torch.int64)
    dout = _bf(4 * TOKENS, 768)
    dtok, dpos = torch.zeros(32000, 768, device="cuda"), torch.zeros(1024, 768, device="cuda")
    return lambda: K.embedding_backward(ids, dout, dtok, dpos, 1024), 0, dout.numel() * 2


def _ew(op: int, dtype: torch.dtype):
    n = 1 << 26
    a = torch.randn(n, device="cuda").to(dtype)
    b = torch.randn(n, device="cuda").to(dtype)
    return lambda: K.ew_binary(op, a, b), 0, 3 * n * a.element_size()


def _case_adamw():
    n = 32 << 20
    p32 = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)

    def run():
        K.adamw_(p32, g, m, v, p16, lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, decoupled=True)

    return run, 0, n * (4 * 4 + 3 * 4 + 2)


def _case_colsum():
    x = _bf(TOKENS, 3072)
    out = torch.zeros(3072, device="cuda")
    return lambda: K.colsum_accum(x, out), 0, x.numel() * 2


def _conv_inputs():
    """3x3 conv, 64 -> 64 channels, 56 x 56, batch 32, stride 1, pad 1 (fp32)."""
    x = torch.randn(32, 64, 56, 56, device="cuda")
    w = torch.randn(64, 64, 3, 3, device="cuda") * 0.05
    b = torch.randn(64, device="cuda")
    flops = 2.0 * 32 * 64 * 56 * 56 * 64 * 9
    return x, w, b, flops


def _case_conv_fwd():
    x, w, b, flops = _conv_inputs()
    return lambda: K.conv2d_fwd(x, w, b, (1, 1), (1, 1)), flops, 2 * x.numel() * 4


def _case_conv_bwd():
    x, w, b, flops = _conv_inputs()
    dy = torch.randn_like(x)
    return lambda: K.conv2d_bwd(dy, x, w, (1, 1), (1, 1), True), 2 * flops, 3 * x.numel() * 4


def _torch_mm_case(m: int, n: int, k: int):
    """Library comparison (not this framework's kernel): torch.matmul bf16,
    i.e. cuBLAS, on the same shape as the named GEMM case."""
    def case():
        a, w = _bf(m, k, scale=0.02), _bf(n, k, scale=0.02)
        return lambda: torch.matmul(a, w.t()), 2.0 * m * n * k, 0
    return case


CASES: dict[str, Callable] = {
    "torch_mm_fwd_qkv": _torch_mm_case(TOKENS, 2304, 768),
    "torch_mm_fc1": _torch_mm_case(TOKENS, 3072, 768),
    "torch_mm_8192": _torch_mm_case(8192, 8192, 8192),
    "conv_fwd": _case_conv_fwd,
    "conv_bwd": _case_conv_bwd,
    "gemm_fwd": _case_gemm_fwd,
    "gemm_fwd_gelu": _case_gemm_fwd_gelu,
    "gemm_dgrad_dgelu": _case_gemm_dgrad_dgelu,
    "gemm_resid_o": _resid_case(768, 768),
    "gemm_resid_fc2": _resid_case(768, 3072),
    "gemm_resid_o_bn128": _resid_variant(128, 0),
    "gemm_resid_o_pair": _resid_variant(256, 1),
    "gemm_o_plain": _plain_case(768, 768, -1),
    "gemm_o_plain_single": _plain_case(768, 768, 0),
    "wgrad_o_split8": _wgrad_split_case(768, 768, 8),
    "wgrad_o_split16": _wgrad_split_case(768, 768, 16),
    "wgrad_qkv_split4": _wgrad_split_case(2304, 768, 4),
    "gemm_wgrad": _case_gemm_wgrad,
    "gemm_8192": _case_gemm_8192,
    # every weight gradient of the 125M step (16384 tokens): fc1, fc2, out-proj, tied head
    "wgrad_fc1": _wgrad_case(3072, 768),
    "wgrad_fc2": _wgrad_case(768, 3072),
    "wgrad_o": _wgrad_case(768, 768),
    "wgrad_head": _wgrad_case(32000, 768),
    "attn_fwd": _case_attn_fwd,
    "attn_fwd16": _case_attn_fwd16,
    "attn_bwd16": _case_attn_bwd16,
    "attn_bwd": _case_attn_bwd,
    "rmsnorm_fwd": _case_rmsnorm_fwd,
    "rmsnorm_bwd": _case_rmsnorm_bwd,
    "softmax_ce": _case_softmax_ce,
    "embedding_fwd": _case_embedding_fwd,
    "embedding_bwd": _case_embedding_bwd,
    "add_bf16": lambda: _ew(K.OP_ADD, torch.bfloat16),
    "mul_bf16": lambda: _ew(K.OP_MUL, torch.bfloat16),
    "add_fp16": lambda: _ew(K.OP_ADD, torch.float16),
    "mul_fp16": lambda: _ew(K.OP_MUL, torch.float16),
    "add_fp32": lambda: _ew(K.OP_ADD, torch.float32),
    "mul_fp32": lambda: _ew(K.OP_MUL, torch.float32),
    "adamw": _case_adamw,
    "colsum": _case_colsum,
}


def time_case(fn: Callable[[], object], iters: int = 20) -> float:
    """Milliseconds per launch, CUDA events on the current stream after 3 warm-ups."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


TRACE_EVENTS = ["start", "qdEmpty", "qdStored", "mmaS", "mmaGrads", "sFull", "sRegs", "math", "pFull", "dqFull",
                "dqDone", "epiStart", "epiEnd", "kvFull"]


def trace_attn_bwd(blocks=(0, 3, 6)) -> str:
    """Run the attention backward of the 125M step (16 x 1024 tokens) once with clock stamps."""
    qkv, o, lse, (B, T, H, D) = _attn_inputs(B=16)
    do = _bf(B * T, H * D)
    nblk = (T + 127) // 128
    buf = torch.zeros(nblk * 16 * 64, dtype=torch.int64, device="cuda")
    for _ in range(3):
        K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True)
    torch.cuda.synchronize()
    K.core().set_attn_bwd_trace(buf.data_ptr())
    try:
        K.flash_attn_qkv_backward(qkv, o, lse, do, B, T, H, D, True)
        torch.cuda.synchronize()
    finally:
        K.core().set_attn_bwd_trace(0)
    tr = buf.view(nblk, 16, 64).cpu()
    out = []
    for blk in blocks:
        if blk >= nblk:
            continue
        t0 = int(tr[blk, 0, 0])
        steps = nblk - blk
        out.append(f"key block {blk}: {steps} query steps; kvFull {int(tr[blk, 13, 0]) - t0}, "
                   f"epiStart {int(tr[blk, 11, 0]) - t0}, epiEnd {int(tr[blk, 12, 0]) - t0}")
        out.append("  step " + " ".join(f"{n:>8s}" for n in TRACE_EVENTS[1:11]))
        for t in range(min(steps, 64)):
            out.append(f"  {t:4d} " + " ".join(f"{int(tr[blk, e, t]) - t0:8d}" for e in range(1, 11)))
    return "\n".join(out)


FWD_TRACE_EVENTS = ["start", "qFull", "kFull", "issueS", "issuePV", "sFullA", "sRegsA", "expA", "oDoneA", "pFullA",
                    "sFullB", "pFullB", "epiStart", "epiEnd"]


def trace_attn_fwd(ctas=(0, 2)) -> str:
    """Run the attention forward of the 125M step (16 x 1024 tokens) once with
    per-key-block clock stamps (tile A = the CTA's first 128 queries)."""
    qkv, _, _, (B, T, H, D) = _attn_inputs(B=16)
    nct = (T + 255) // 256
    buf = torch.zeros(nct * 16 * 64, dtype=torch.int64, device="cuda")
    for _ in range(3):
        K.flash_attn_qkv(qkv, B, T, H, D, True)
    torch.cuda.synchronize()
    K.core().set_attn_fwd_trace(buf.data_ptr())
    try:
        K.flash_attn_qkv(qkv, B, T, H, D, True)
        torch.cuda.synchronize()
    finally:
        K.core().set_attn_fwd_trace(0)
    tr = buf.view(nct, 16, 64).cpu()
    out = []
    for c in ctas:
        if c >= nct:
            continue
        t0 = int(tr[c, 0, 0])
        m_block = nct - 1 - c  # the kernel runs the longest rows first
        n_b = min((T + 127) // 128, 2 * m_block + 2)
        out.append(f"CTA {c} (queries {m_block * 256}..{m_block * 256 + 255}): {n_b} key blocks; "
                   f"qFull {int(tr[c, 1, 0]) - t0}, epiStart {int(tr[c, 12, 0]) - t0}, epiEnd {int(tr[c, 13, 0]) - t0}")
        out.append("  blk  " + " ".join(f"{n:>8s}" for n in FWD_TRACE_EVENTS[2:12]))
        for j in range(n_b):
            out.append(f"  {j:4d} " + " ".join(f"{int(tr[c, e, j]) - t0:8d}" if int(tr[c, e, j]) else f"{'-':>8s}"
                                             for e in range(2, 12)))
    return "\n".join(out)


GEMM_TRACE_EVENTS = ("prodStart", "prodLast", "mmaAccFree", "mmaFirstFull", "mmaCommit", "epiFull", "epiRelease",
                     "epiDone", "ld0", "ld1", "ld2", "ld3", "math0", "math1", "math2", "math3", "st0", "st1", "st2",
                     "st3")


def trace_gemm(name: str) -> str:
    """Run one GEMM case with the single-CTA kernel's per-unit clock stamps
    (CTA 0; build with UNDERHFS_GEMM_TRACE=1): SM cycles from the first stamp
    for each unit the CTA processed."""
    fn, _, _ = CASES[name]()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    buf = torch.zeros(len(GEMM_TRACE_EVENTS) * 16, dtype=torch.int64, device="cuda")
    K.core().set_gemm_trace(buf.data_ptr())
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        K.core().set_gemm_trace(0)
    tr = buf.view(len(GEMM_TRACE_EVENTS), 16).cpu()
    nz = tr[tr != 0]
    if nz.numel() == 0:
        return f"{name}: no stamps (single-CTA kernel not used, or a build without UHFS_GEMM_TRACE)"
    t0 = int(nz.min())
    out = [f"{name}: CTA 0, SM cycles from its first stamp",
           "  unit " + " ".join(f"{e:>7s}" for e in GEMM_TRACE_EVENTS)]
    for u in range(16):
        if int(tr[:, u].abs().sum()) == 0:
            continue
        out.append(f"  {u:4d} " + " ".join(f"{int(tr[e, u]) - t0:7d}" if int(tr[e, u]) else f"{'-':>7s}"
                                           for e in range(len(GEMM_TRACE_EVENTS))))
    return "\n".join(out)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", nargs="+", choices=sorted(CASES) + ["all"], help="one or more cases, or all")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="print CUDA-event time per launch")
    ap.add_argument("--trace", action="store_true",
                    help="attn_fwd / attn_bwd / gemm_*: print the kernel's clock stamps (trace builds)")
    args = ap.parse_args(argv)
    torch.manual_seed(0)
    if args.trace:
        if any(c.startswith("gemm_") for c in args.case):
            for c in args.case:
                print(trace_gemm(c))
            st = K.core().device_status(True)
            print("ok" if st["code"] == 0 else f"device status {st}")
            return 0 if st["code"] == 0 else 1
        if len(args.case) != 1 or args.case[0] not in ("attn_bwd", "attn_fwd"):
            ap.error("--trace is available for attn_fwd, attn_bwd and the gemm_* cases")
        print(trace_attn_bwd() if args.case[0] == "attn_bwd" else trace_attn_fwd())
        st = K.core().device_status(True)
        print("ok" if st["code"] == 0 else f"device status {st}")
        return 0 if st["code"] == 0 else 1
    names = sorted(CASES) if "all" in args.case else args.case
    for name in names:
        fn, flops, nbytes = CASES[name]()
        if args.time:
            ms = time_case(fn)
            rate = f"{flops / ms / 1e9:.0f} TFLOP/s" if flops else f"{nbytes / ms / 1e6:.0f} GB/s"
            print(f"{name}: {ms * 1e3:.1f} us/launch, {rate}", flush=True)
        else:
            for _ in range(args.iters):
                fn()
        torch.cuda.synchronize()
        st = K.core().device_status(True)
        if st["code"] != 0:
            print(f"{name}: device status {st}", file=sys.stderr)
            return 1
        del fn
        torch.cuda.empty_cache()
    print("ok")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
