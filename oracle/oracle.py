"""CPU oracle for the paged-KV hot path — TEST INFRASTRUCTURE ONLY.

Used by tests/, by ``__graft_entry__.smoke()`` as the checker and by
bench.py's CPU-baseline leg; the product package never imports it.

What it restates (reference = src/triton_kernels/paged_kv.py):
  decode        -> oracle/pkv_oracle.c, the 3-pass _paged_attention_decode_kernel
                   (:63-251), called through ctypes, multithreaded with pthreads;
  decode_numpy  -> the same three passes in numpy, for cross-checking the C
                   restatement on small cases;
  append        -> _paged_kv_update_kernel (:253-319): slot = pre-append length;
  append_prompt -> the prefill scatter of _prefill_paged_cache (:576-586);
  gather        -> the decode kernel's addressing (:98-131) written densely;
  sample_top_p  -> _sample_tokens / _apply_top_p (:418-450): scaled logits in the
                   logits dtype, stable descending sort, running probability,
                   nucleus cut, then the draw for a given uniform by the inverse
                   CDF of the kept tokens in index order (the CUDA op's draw);
  nucleus       -> the kept-token mask of that rule alone, with the exact
                   probabilities (pinned to the reference's own _apply_top_p
                   by tests/golden/sampling_*.npz);
  rmsnorm       -> the arithmetic of the reference's _rmsnorm_kernel
                   (src/triton_kernels/fused_ops.py:34-77): fp32 sum of squares,
                   x * rsqrt(mean + eps) rounded to bf16, times the weight,
                   rounded to bf16 (pinned by tests/golden/rmsnorm_*.npz).
The byte-moving functions work on raw-bit numpy views, so they are exact for
every dtype. Parity of this oracle with the reference itself is pinned by
tests/golden/ (fixtures produced by running the reference's own kernels).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libpkv_oracle.so"

_DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_RAW = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}


def build(force: bool = False) -> Path:
    """Compile oracle/libpkv_oracle.so with gcc (via oracle/Makefile)."""
    src = HERE / "pkv_oracle.c"
    if force or not LIB_PATH.exists() or src.stat().st_mtime > LIB_PATH.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "all"], check=True)
    return LIB_PATH


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        lib = C.CDLL(str(LIB_PATH))
        i32, vp, i64p = C.c_int32, C.c_void_p, C.POINTER(C.c_int64)
        lib.oracle_decode.restype = C.c_int
        lib.oracle_decode.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32,
                                      i64p, i64p, i64p, i64p, i32, i32, C.c_float, i32]
        lib.oracle_max_threads.restype = C.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().oracle_max_threads())


def _i64(vals):
    vals = [int(v) for v in vals]
    return (C.c_int64 * len(vals))(*vals)


def _cpu(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        raise ValueError("the oracle takes CPU tensors")
    return t


def decode(q, k_cache, v_cache, block_tables, context_lens, scale=None, nthreads=0) -> torch.Tensor:
    """fp32 [B, Hq, D] decode attention by the C restatement (any strides, f32/bf16/f16)."""
    for t in (q, k_cache, v_cache, block_tables, context_lens):
        _cpu(t)
    batch, hq, head_dim = q.shape
    num_blocks, hkv, bs, _ = k_cache.shape
    assert k_cache.stride() == v_cache.stride()
    bt = block_tables.to(torch.int32)
    ctx = context_lens.to(torch.int32).contiguous()
    out = torch.zeros((batch, hq, head_dim), dtype=torch.float32)
    if scale is None:
        scale = 1.0 / float(np.sqrt(head_dim))
    rc = _load().oracle_decode(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), ctx.data_ptr(),
        out.data_ptr(), batch, hq, hkv, head_dim, bs, num_blocks, bt.shape[1],
        _i64(q.stride()), _i64(k_cache.stride()), _i64(bt.stride()), _i64(out.stride()),
        _DT[q.dtype], _DT[k_cache.dtype], float(scale), int(nthreads),
    )
    if rc != 0:
        raise ValueError(f"oracle_decode rejected the arguments ({rc})")
    return out


def decode_numpy(q, k_cache, v_cache, block_tables, context_lens, scale=None) -> np.ndarray:
    """The same three passes in numpy (small cases only)."""
    qf = q.float().numpy()
    kf = k_cache.float().numpy()
    vf = v_cache.float().numpy()
    bt = block_tables.numpy().astype(np.int64)
    ctx = context_lens.numpy().astype(np.int64)
    batch, hq, head_dim = qf.shape
    num_blocks, hkv, bs, _ = kf.shape
    group = hq // hkv
    if scale is None:
        scale = np.float32(1.0 / np.sqrt(head_dim))
    out = np.zeros((batch, hq, head_dim), dtype=np.float32)
    cap = bt.shape[1] * bs
    for b in range(batch):
        n = int(min(max(ctx[b], 0), cap))
        if n == 0:
            continue
        pos = np.arange(n)
        pages = bt[b, pos // bs]
        ok = (pages >= 0) & (pages < num_blocks)
        pos, pages = pos[ok], pages[ok]
        for h in range(hq):
            kv = h // group
            K = kf[pages, kv, pos % bs, :]
            V = vf[pages, kv, pos % bs, :]
            logits = (K @ qf[b, h]).astype(np.float32) * np.float32(scale)
            m = logits.max()
            w = np.exp(logits - m).astype(np.float32)
            s = w.sum(dtype=np.float32)
            out[b, h] = (w @ V) / max(s, np.float32(1e-6))
    return out


def _raw(t: torch.Tensor) -> np.ndarray:
    """Raw-bit numpy view of a CPU tensor (bf16 has no numpy dtype)."""
    return _cpu(t).view(_RAW[t.dtype]).numpy()


def append(k_new, v_new, k_cache, v_cache, block_tables, context_lens) -> None:
    """In-place: cache[page(ctx_b), h, ctx_b % bs, :] = new[b, h, :] (paged_kv.py:277-319)."""
    kc, vc = _raw(k_cache), _raw(v_cache)
    kn, vn = _raw(k_new), _raw(v_new)
    bt = block_tables.numpy()
    ctx = context_lens.numpy()
    bs = k_cache.shape[2]
    for b in range(kn.shape[0]):
        pos = int(ctx[b])
        page = int(bt[b, pos // bs])
        kc[page, :, pos % bs, :] = kn[b]
        vc[page, :, pos % bs, :] = vn[b]


def append_prompt(k, v, k_cache, v_cache, block_tables, start_pos=None, lens=None) -> None:
    """In-place prompt scatter of k/v [B, H, T, D] (paged_kv.py:576-586)."""
    kc, vc = _raw(k_cache), _raw(v_cache)
    ks, vs = _raw(k), _raw(v)
    bt = block_tables.numpy()
    batch, _, seq_len, _ = ks.shape
    bs = k_cache.shape[2]
    for b in range(batch):
        n = seq_len if lens is None else int(lens[b])
        s0 = 0 if start_pos is None else int(start_pos[b])
        for t in range(n):
            pos = s0 + t
            page = int(bt[b, pos // bs])
            kc[page, :, pos % bs, :] = ks[b, :, t, :]
            vc[page, :, pos % bs, :] = vs[b, :, t, :]


def gather(k_cache, v_cache, block_tables, context_lens, max_tokens=None):
    """Dense K, V [B, H, T, D]; zero beyond context_lens[b]."""
    kc, vc = _raw(k_cache), _raw(v_cache)
    bt = block_tables.numpy()
    ctx = context_lens.numpy()
    num_blocks, heads, bs, head_dim = kc.shape
    batch = bt.shape[0]
    if max_tokens is None:
        max_tokens = bt.shape[1] * bs
    ko = np.zeros((batch, heads, max_tokens, head_dim), dtype=kc.dtype)
    vo = np.zeros_like(ko)
    for b in range(batch):
        n = min(int(ctx[b]), max_tokens, bt.shape[1] * bs)
        for t in range(n):
            page = int(bt[b, t // bs])
            ko[b, :, t, :] = kc[page, :, t % bs, :]
            vo[b, :, t, :] = vc[page, :, t % bs, :]
    dt = k_cache.dtype
    return torch.from_numpy(ko).view(dt), torch.from_numpy(vo).view(dt)


if __name__ == "__main__":  # pragma: no cover
    print(build(force=True), max_threads(), os.cpu_count())


def nucleus(logits, temperature: float, top_p: float):
    """Exact-rule nucleus of each row: (kept bool [B, V], scaled float64 [B, V],
    p float64 [B, V]). scaled = logits / max(T, 1e-6) rounded to the logits dtype
    (paged_kv.py:446); p = softmax(scaled) in float64; in descending order with
    ties in index order, a token is kept while the running probability including
    it is <= top_p (paged_kv.py:426-429), the first always (:428); top_p >= 1
    keeps every token."""
    lg = _cpu(logits)
    scaled = (lg.float() / max(float(temperature), 1e-6)).to(lg.dtype).double().numpy()
    B, V = scaled.shape
    kept = np.ones((B, V), dtype=bool)
    p = np.exp(scaled - scaled.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    if top_p < 1.0:
        for b in range(B):
            order = np.argsort(-scaled[b], kind="stable")
            keep_sorted = np.cumsum(p[b, order]) <= top_p
            keep_sorted[0] = True
            kept[b] = False
            kept[b, order[keep_sorted]] = True
    return kept, scaled, p


def rmsnorm(x, weight, eps: float, cast_rounding: str = "rne") -> torch.Tensor:
    """bf16 [rows, hidden]: the reference _rmsnorm_kernel's arithmetic in numpy
    (fused_ops.py:48-77): s = sum of fp32 squares, inv = 1 / sqrt(s / n + eps) in
    fp32, normed = bf16(x * inv), y = bf16(normed * w). cast_rounding is the
    rounding of the kernel's fp32 -> bf16 cast of `normed` (:73): "rne" (to
    nearest even, compiled Triton's default on the GPU) or "rtz" (toward zero,
    what Triton's CPU interpreter does)."""
    xf = _cpu(x).float().numpy()
    wf = _cpu(weight).float().numpy()
    n = np.float32(xf.shape[1])
    s = (xf * xf).sum(axis=1, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(s / n + np.float32(eps))).astype(np.float32)
    prod = (xf * inv[:, None]).astype(np.float32)
    if cast_rounding == "rtz":
        normed = torch.from_numpy((prod.view(np.int32) & np.int32(~0xFFFF)).view(np.float32))
    elif cast_rounding == "rne":
        normed = torch.from_numpy(prod).to(torch.bfloat16).float()
    else:
        raise ValueError(f"cast_rounding must be 'rne' or 'rtz', got {cast_rounding!r}")
    return (normed * torch.from_numpy(wf)).to(torch.bfloat16)


def sample_top_p(logits, temperature: float, top_p: float, uniforms):
    """Token per row and the two margins that decide it, for uniforms u in [0, 1).

    Follows paged_kv.py:418-450: scaled = logits / max(T, 1e-6) rounded to the
    logits dtype, probabilities softmax(scaled) (here in float64), the sorted
    order descending with ties in index order (a stable sort), tokens kept
    while their running probability is <= top_p, the first always kept. The
    draw inverts the CDF of the kept tokens in that sorted order at
    u * kept mass, as a multinomial draw over the sorted probabilities does.
    Returns (tokens int64 [B], cut_margin [B], draw_margin [B]): the distance
    of the running probability from top_p at the cut and of the target from
    the nearest CDF step, so a test can skip rows that float rounding decides.
    """
    lg = _cpu(logits)
    scaled = (lg.float() / max(float(temperature), 1e-6)).to(lg.dtype).double().numpy()
    u = np.asarray(_cpu(torch.as_tensor(uniforms)).double())
    B, V = scaled.shape
    toks = np.zeros(B, dtype=np.int64)
    cut_margin = np.full(B, np.inf)
    draw_margin = np.full(B, np.inf)
    for b in range(B):
        x = scaled[b]
        p = np.exp(x - x.max())
        p /= p.sum()
        order = np.argsort(-x, kind="stable")
        run = np.cumsum(p[order])
        keep_sorted = run <= top_p if top_p < 1.0 else np.ones(V, dtype=bool)
        keep_sorted[0] = True
        if top_p < 1.0:
            cut_margin[b] = float(np.min(np.abs(run - top_p)))
        idx = order[keep_sorted]
        cdf = np.cumsum(p[idx])
        target = u[b] * cdf[-1]
        j = int(np.searchsorted(cdf, target, side="right"))
        toks[b] = idx[min(j, len(idx) - 1)]
        draw_margin[b] = float(np.min(np.abs(cdf - target)))
    return torch.from_numpy(toks), cut_margin, draw_margin
