"""Oracle for the fused lm_head cross-entropy head — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or the timed CPU
baseline. The product path (``rus_b200``) never imports it and has no CPU
fallback.

Contents
--------
``eager_head``      The reference's eager formula (what the north-star parity is
                    defined against): full logits ``F.linear(X, W)`` in the input
                    dtype, ``.float()``, cross-entropy with ignore_index -100,
                    loss = sum(nll) / denom, entropy = logsumexp(z) - sum(softmax(z) z),
                    argmax(z); gradients by autograd through the same graph
                    (fp16/bf16 gradient of the logits, like the GPU eager path)
                    or, with ``grad_mode="fp32"``, the exact fp32 gradient.
                    Follows solution/test_kernels.py:204-216 (the reference's own
                    known-answer test), harness/eval_adapter.py:57-62 and the
                    denominator rule of solution/ops.py:268-277.
``chunked_restatement``
                    A numpy restatement of the reference's chunked algorithm:
                    pass 1 online (m, s, w, argmax, target) per vocab chunk
                    (solution/kernels.py:480-516, driven by ops.py:216-251),
                    finish (kernels.py:534-565), loss (ops.py:268-277), and the
                    2^16-prescaled fp16 gradient pass with an fp16 dX accumulator
                    (ops.py:280-338, kernels.py:517-531).
``part_merge_np`` / ``parts_of_shard``
                    The per-token partial record (m, s, w, best, idx, zy) of a
                    vocab range and its merge — the statistics protocol the
                    vocab-sharded head gathers across GPUs.
``rms_norm_ref``    The reference's final RMSNorm as differentiable torch ops with its
                    casting order (solution/kernels.py:124-164): rstd in fp32, the
                    normalised row rounded to the input dtype, times the weight,
                    rounded again; ``rms_norm_bwd_ref`` its backward formula
                    (kernels.py:167-190).
``pack_restatement`` / ``scatter_restatement``
                    Plain-Python loops of the packing around the head: label
                    shift, keep mask and compaction (solution/ops.py:1107-1127),
                    and the scatter back with the mean-entropy filler
                    (ops.py:1151-1164).

Parity pin: tests/golden/ holds outputs of the reference's own ``chunked_lm_head``
(run on CPU through Triton's interpreter, tests/golden/make_golden.py) on the
reference test's inputs and on extra edge cases; tests/test_oracle.py checks
this module against them.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

IGNORE = -100
PRESCALE_GRAD = 65536.0  # the reference's fp16 prescale (ops.py:171)


def denominator(labels: torch.Tensor, num_items_in_batch=None) -> float:
    """ops.py:268-277: num_items_in_batch if given, else #valid labels; clamped to >= 1."""
    if num_items_in_batch is not None:
        d = float(num_items_in_batch.item() if isinstance(num_items_in_batch, torch.Tensor) else num_items_in_batch)
    else:
        d = float((labels != IGNORE).sum().item())
    return max(d, 1.0)


def eager_head(hidden: torch.Tensor, labels: torch.Tensor, weight: torch.Tensor, num_items_in_batch=None,
               grads: bool = True, grad_mode: str = "eager") -> dict:
    """The reference eager path on whatever device the tensors live on.

    hidden [N, H], labels [N], weight [V, H] (same 16-bit dtype). Returns a dict of
    loss, nll, entropy, argmax, lse, logits_max and, if ``grads``, dX and dW."""
    h = hidden.detach().reshape(-1, hidden.shape[-1])
    y = labels.reshape(-1).to(torch.int64)
    w = weight.detach()
    denom = denominator(y, num_items_in_batch)
    out: dict = {"denom": denom}
    if grads and grad_mode == "eager":
        h = h.clone().requires_grad_(True)
        w = w.clone().requires_grad_(True)
    with torch.set_grad_enabled(grads and grad_mode == "eager"):
        logits16 = F.linear(h, w)  # input dtype, like the reference's GPU eager path
        z = logits16.float()
        nll = F.cross_entropy(z, y, ignore_index=IGNORE, reduction="none")
        loss = nll.sum() / denom
    with torch.no_grad():
        zd = z.detach()
        lse = torch.logsumexp(zd, dim=-1)
        probs = torch.softmax(zd, dim=-1)
        ent = lse - (probs * zd).sum(-1)
        arg = zd.argmax(dim=-1)
    out.update(loss=loss.detach(), nll=nll.detach(), entropy=ent, argmax=arg, lse=lse)
    if not grads:
        return out
    if grad_mode == "eager":
        loss.backward()
        out["dX"] = h.grad.detach()
        out["dW"] = w.grad.detach()
    elif grad_mode == "fp32":
        with torch.no_grad():
            g = probs.clone()
            valid = y != IGNORE
            idx = torch.nonzero(valid).squeeze(-1)
            g[idx, y[idx]] -= 1.0
            g[~valid] = 0.0
            g /= denom
            out["dX"] = g @ weight.detach().float()
            out["dW"] = g.t() @ hidden.detach().reshape(-1, hidden.shape[-1]).float()
    else:
        raise ValueError(grad_mode)
    return out


def _np16(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        # numpy has no bfloat16: carry the exact values in fp32
        return t.detach().float().cpu().numpy()
    return t.detach().cpu().numpy()


def _round(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.float16:
        return x.astype(np.float16).astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def chunked_restatement(hidden: torch.Tensor, labels: torch.Tensor, weight: torch.Tensor, num_items_in_batch=None,
                        v_chunk: int = 8192, block_v: int = 1024, grad_loss: float = 1.0) -> dict:
    """Restatement of the reference's chunked head (ops.py:179-338, kernels.py:453-565) in numpy.

    Logit chunks are fp32-accumulated and rounded to the input dtype like the
    reference's fp16 ``torch.mm`` output (ops.py:231); the gradient is formed as
    ``(exp(z - lse) - onehot) * 2^16 / denom`` rounded to the input dtype
    (kernels.py:517-531) and accumulated chunk by chunk into an input-dtype dX
    buffer (ops.py:283, 320), then rescaled by grad_loss / 2^16 (ops.py:337-338)."""
    dt = hidden.dtype
    h = _np16(hidden.reshape(-1, hidden.shape[-1])).astype(np.float32)
    w_all = _np16(weight).astype(np.float32)
    y = labels.reshape(-1).to(torch.int64).cpu().numpy()
    n, _ = h.shape
    v = w_all.shape[0]
    f32 = np.float32
    m = np.full(n, -1.0e30, f32)
    s = np.zeros(n, f32)
    wsum = np.zeros(n, f32)
    zy = np.zeros(n, f32)
    best_val = np.full(n, -1.0e30, f32)
    best_idx = np.zeros(n, np.int64)
    n_chunks = (v + v_chunk - 1) // v_chunk
    for c in range(n_chunks):
        c0, c1 = c * v_chunk, min((c + 1) * v_chunk, v)
        z = _round(h @ w_all[c0:c1].T, dt)
        cols = c1 - c0
        for t0 in range(0, cols, block_v):
            t1 = min(t0 + block_v, cols)
            tile = z[:, t0:t1]
            tile_max = tile.max(axis=1)
            upd = tile_max > best_val  # strict: earlier tiles win ties (kernels.py:495)
            best_idx[upd] = c0 + t0 + tile.argmax(axis=1)[upd]
            best_val[upd] = tile_max[upd]
            m_new = np.maximum(m, tile_max)
            alpha = np.exp(m - m_new)
            e = np.exp(tile - m_new[:, None])
            s = s * alpha + e.sum(axis=1)
            wsum = wsum * alpha + (e * tile).sum(axis=1)
            m = m_new
        inside = (y >= c0) & (y < c1)
        zy[inside] = z[np.nonzero(inside)[0], y[inside] - c0]
    lse = m + np.log(s)
    ent = lse - wsum / s
    valid = y != IGNORE
    nll = np.where(valid, lse - zy, 0.0).astype(f32)
    denom = denominator(torch.from_numpy(y), num_items_in_batch)
    loss = f32(nll.sum(dtype=np.float64) / denom)
    # gradient pass: reversed chunks, prescaled G in the input dtype, dX accumulator in the input dtype
    grad_scale = PRESCALE_GRAD / denom
    dxp = np.zeros_like(h)
    for c in range(n_chunks - 1, -1, -1):
        c0, c1 = c * v_chunk, min((c + 1) * v_chunk, v)
        z = _round(h @ w_all[c0:c1].T, dt)
        prob = np.exp(z - lse[:, None])
        onehot = np.zeros_like(prob)
        inside = (y >= c0) & (y < c1)
        onehot[np.nonzero(inside)[0], y[inside] - c0] = 1.0
        g = _round((prob - onehot) * np.where(valid, grad_scale, 0.0)[:, None], dt)
        dxp = _round(dxp + g @ w_all[c0:c1], dt)
    scale = _round(np.array([grad_loss / PRESCALE_GRAD], f32), dt)[0]
    dx = _round(dxp * scale, dt)
    return dict(loss=loss, nll=nll, entropy=ent.astype(f32), argmax=best_idx, lse=lse.astype(f32), dX=dx,
                denom=denom)


# ----------------------------------------------------------- partial records

PART_FIELDS = ("m", "s", "w", "best", "idx", "zy")


def parts_of_shard(hidden: torch.Tensor, labels: torch.Tensor, weight_shard: torch.Tensor, vocab_offset: int) -> dict:
    """Per-token partial record of one vocab shard (logits rounded to the input dtype).

    s = sum exp(z - m), w = sum exp(z - m)(z - m), best/idx = max logit and its lowest
    global id, zy = target logit or -inf when the target is outside the shard."""
    z = F.linear(hidden.detach().reshape(-1, hidden.shape[-1]), weight_shard.detach()).float().cpu().numpy()
    y = labels.reshape(-1).to(torch.int64).cpu().numpy().astype(np.int64)
    m = z.max(axis=1)
    d = z - m[:, None]
    e = np.exp(d.astype(np.float64))
    v = z.shape[1]
    yl = y - vocab_offset
    inside = (y != IGNORE) & (yl >= 0) & (yl < v)
    zy = np.full(len(y), -np.inf)
    zy[inside] = z[np.nonzero(inside)[0], yl[inside]]
    return dict(m=m.astype(np.float64), s=e.sum(1), w=(e * d).sum(1), best=m.astype(np.float64),
                idx=z.argmax(axis=1).astype(np.int64) + vocab_offset, zy=zy)


def part_merge_np(records: list[dict]) -> dict:
    """Merge per-token partial records of disjoint vocab ranges (float64)."""
    mx = np.max(np.stack([r["m"] for r in records]), axis=0)
    s = np.zeros_like(mx)
    w = np.zeros_like(mx)
    best = np.full_like(mx, -np.inf)
    idx = np.full(mx.shape, np.iinfo(np.int64).max, dtype=np.int64)
    zy = np.full_like(mx, -np.inf)
    for r in records:
        d = r["m"] - mx
        a = np.exp(d)
        s += a * r["s"]
        w += a * (r["w"] + d * r["s"])
        take = (r["best"] > best) | ((r["best"] == best) & (r["idx"] < idx))
        best = np.where(take, r["best"], best)
        idx = np.where(take, r["idx"], idx)
        zy = np.maximum(zy, r["zy"])
    return dict(m=mx, s=s, w=w, best=best, idx=idx, zy=zy)


def finish_np(rec: dict, labels: torch.Tensor, num_items_in_batch=None) -> dict:
    """lse = m + ln s, entropy = ln s - w / s, nll = lse - zy (0 for ignored), loss = sum / denom."""
    y = labels.reshape(-1).to(torch.int64).cpu().numpy()
    ln_s = np.log(rec["s"])
    lse = rec["m"] + ln_s
    ent = ln_s - rec["w"] / rec["s"]
    nll = np.where(y != IGNORE, lse - rec["zy"], 0.0)
    denom = denominator(torch.from_numpy(y), num_items_in_batch)
    return dict(lse=lse, entropy=ent, nll=nll, argmax=rec["idx"], loss=nll.sum() / denom, denom=denom)


# ------------------------------------------------------------ comparisons

def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def argmax_mismatch_ok(ours: torch.Tensor, ref: torch.Tensor, logits32: torch.Tensor, dtype: torch.dtype,
                       tol: float = 1e-3) -> torch.Tensor:
    """Per-token: True where ours == ref, or where the two candidates' fp32 logits lie
    within max(tol, one ulp of the input dtype at that magnitude) — the north-star rule
    'bit-exact except where the top-2 logits lie within 1e-3', widened to the rounding
    step the reference's own fp16/bf16 logits have."""
    ours = ours.cpu().long()
    ref = ref.cpu().long()
    z = logits32.cpu().float()
    rows = torch.arange(z.shape[0])
    zo = z[rows, ours]
    zr = z[rows, ref]
    mag = torch.maximum(zo.abs(), zr.abs())
    mant = 10 if dtype == torch.float16 else 7
    ulp = torch.exp2(torch.floor(torch.log2(mag.clamp_min(1e-30))) - mant)
    return (ours == ref) | ((zo - zr).abs() <= torch.maximum(torch.full_like(ulp, tol), ulp))


def argmax_tie_report(ours: torch.Tensor, ref: torch.Tensor, logits32: torch.Tensor, dtype: torch.dtype,
                      tol: float = 1e-3) -> dict:
    """Per-token argmax agreement, by the rule that accepts each token:

    ``exact``     ours == ref;
    ``strict``    mismatch whose two candidates' fp32 logits lie within ``tol`` (the north-star rule);
    ``widened``   mismatch accepted only by the one-ulp widening of ``argmax_mismatch_ok``;
    ``rejected``  mismatch outside both;
    ``not_top``   accepted mismatches where a candidate is not at the top of its row, i.e. its
                  fp32 logit lies more than one input-dtype ulp (plus ``tol``) below the row's
                  fp32 maximum. Every accepted mismatch must be a real near-tie at the top, so
                  this must be 0.
    Also returns ``ok`` (the per-token mask of argmax_mismatch_ok) and the largest candidate gap."""
    ours = ours.cpu().long()
    ref = ref.cpu().long()
    z = logits32.cpu().float()
    rows = torch.arange(z.shape[0])
    zo = z[rows, ours]
    zr = z[rows, ref]
    zmax = z.max(dim=1).values
    mant = 10 if dtype == torch.float16 else 7
    ulp_of = lambda x: torch.exp2(torch.floor(torch.log2(x.abs().clamp_min(1e-30))) - mant)  # noqa: E731
    ulp = ulp_of(torch.maximum(zo.abs(), zr.abs()))
    gap = (zo - zr).abs()
    mism = ours != ref
    strict = mism & (gap <= tol)
    widened = mism & ~strict & (gap <= ulp)
    accepted = strict | widened
    below = zmax - torch.minimum(zo, zr)
    not_top = accepted & (below > ulp_of(zmax) + tol)
    return {"tokens": int(z.shape[0]), "exact": int((~mism).sum()), "strict": int(strict.sum()),
            "widened": int(widened.sum()), "rejected": int((mism & ~accepted).sum()),
            "not_top": int(not_top.sum()), "max_gap": float(gap[mism].max()) if bool(mism.any()) else 0.0,
            "ok": ~mism | accepted}


# -------------------------------------------------------------- generators

def zipf_truncated_lengths(rng: np.random.Generator, rows: int, a: float = 1.2, kmax: int = 512) -> np.ndarray:
    """Row lengths from a Zipf(a) law truncated to 1..kmax: P(k) proportional to k^-a on that support
    (for a = 1.2, kmax = 512 the mean is ~44 tokens, so 64 rows give E[N] ~ 2.8k)."""
    k = np.arange(1, kmax + 1)
    pmf = k ** -a
    return rng.choice(k, size=rows, p=pmf / pmf.sum()).astype(int)


def make_config_inputs(cfg: str, seed: int = 0, device: str = "cpu", n_override: int | None = None):
    """Seeded synthetic inputs for the five BASELINE.json configs (the contest dataset is absent;
    lengths, value distributions and label masks follow the config descriptions).

    Returns (hidden [N,H], labels [N] int64, weight [V,H], meta dict)."""
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    if cfg in ("c1", "c2", "c5"):
        H, V, dt = (896, 151936, torch.float16) if cfg == "c5" else (1536, 151936, torch.float16)
    elif cfg == "c3":
        H, V, dt = 3584, 152064, torch.float16
    elif cfg == "c4":
        H, V, dt = 4096, 128256, torch.bfloat16
    else:
        raise ValueError(cfg)
    w_std = 0.02
    if cfg == "c1":
        lens = np.clip(np.round(rng.lognormal(math.log(140), 0.951, 4)), 16, 512).astype(int)
    elif cfg == "c2":
        lens = np.full(4, 512)
    elif cfg == "c3":
        lens = np.clip(np.round(rng.lognormal(math.log(600), 0.67, 16)), 32, 2048).astype(int)
    elif cfg == "c4":
        lens = np.full(8, 4096)
    else:  # c5: Zipf(1.2) truncated to 1..512 (the pmf renormalised on that support; E[N] ~ 2.8k)
        lens = zipf_truncated_lengths(rng, 64)
        w_std = 12.0 / math.sqrt(H)
    if n_override is not None:
        # keep the row structure but cap the total (parity tests at oracle-friendly sizes)
        scale = n_override / lens.sum()
        lens = np.maximum(1, np.round(lens * scale)).astype(int)
    N = int(lens.sum())
    W = (torch.randn(V, H, generator=g) * w_std).to(dt)
    X = torch.randn(N, H, generator=g)
    if cfg in ("c1", "c2", "c3", "c5"):
        gamma = 1.0 + 0.1 * torch.randn(H, generator=g)  # RMSNorm weight ~ N(1, 0.1)
        X = X * gamma
    X = X.to(dt)
    labels = torch.randint(0, V, (N,), generator=g)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    if cfg == "c1":
        for s0, L in zip(starts, lens):
            labels[s0:s0 + int(0.4 * L)] = IGNORE
    elif cfg in ("c2", "c3"):
        mask = torch.rand(N, generator=g) < 0.10
        labels[mask] = IGNORE
    elif cfg == "c5":
        for r in rng.choice(len(lens), 3, replace=False):
            labels[starts[r]:starts[r] + lens[r]] = IGNORE
        # exact argmax ties on ~1% of tokens: duplicate a W row and align x to it
        n_tie = max(1, N // 100)
        tok = rng.choice(N, n_tie, replace=False)
        for t in tok:
            a, b = (int(v) for v in rng.choice(V, 2, replace=False))
            W[b] = W[a]
            X[t] = (W[a].float() * (40.0 / W[a].float().norm())).to(dt)
    meta = dict(cfg=cfg, N=N, H=H, V=V, dtype=str(dt).replace("torch.", ""), lens=lens.tolist(), seed=seed)
    return X.to(device), labels.to(device), W.to(device), meta


def pack_restatement(labels: torch.Tensor, mask: torch.Tensor | None):
    """solution/ops.py:1107-1127 as loops: shift labels left (last position -100), keep a
    position when attended or labelled, position 0 of every row when nothing is kept;
    returns (shift labels of kept positions, their flat indices, kept count per row)."""
    B, S = labels.shape
    shift = [[IGNORE] * S for _ in range(B)]
    for b in range(B):
        for s in range(S - 1):
            shift[b][s] = int(labels[b, s + 1])
    keep = [[(mask is not None and bool(mask[b, s])) or (mask is None) or shift[b][s] != IGNORE for s in range(S)]
            for b in range(B)]
    if not any(any(r) for r in keep):
        for b in range(B):
            keep[b][0] = True
    idx = [b * S + s for b in range(B) for s in range(S) if keep[b][s]]
    return [shift[i // S][i % S] for i in idx], idx, [sum(r) for r in keep]


def scatter_restatement(total: int, idx: list, nll: list, ent: list, arg: list):
    """solution/ops.py:1151-1164 as loops: kept positions get their values, the others nll 0,
    argmax 0 and the mean entropy of the kept tokens (0 when none)."""
    mean = float(sum(ent)) / len(ent) if ent else 0.0
    full_nll, full_ent, full_arg = [0.0] * total, [mean] * total, [0] * total
    for i, t in enumerate(idx):
        full_nll[t], full_ent[t], full_arg[t] = nll[i], ent[i], arg[i]
    return full_nll, full_ent, full_arg


def rms_norm_ref(h: torch.Tensor, w: torch.Tensor, eps: float = 1e-6):
    """solution/kernels.py:124-164 without residual: (out, rstd); differentiable in h."""
    hf = h.float()
    rstd = torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)
    normed = (hf * rstd).to(h.dtype)
    out = (normed.float() * w.float()).to(h.dtype)
    return out, rstd.squeeze(-1)


def rms_norm_bwd_ref(dy: torch.Tensor, h: torch.Tensor, w: torch.Tensor, rstd: torch.Tensor) -> torch.Tensor:
    """solution/kernels.py:167-190 without residual: dh = (w dy - x_hat mean(x_hat w dy)) rstd."""
    x_hat = h.float() * rstd[..., None]
    wdy = w.float() * dy.float()
    c1 = (x_hat * wdy).mean(-1, keepdim=True)
    return ((wdy - x_hat * c1) * rstd[..., None]).to(h.dtype)
