"""Training-path oracle: the reference's fine-tuning step restated for the CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  The floating-point training kernels are checked against a
PyTorch fp32 restatement of the reference's model with autograd for the gradients; the loss, the optimizer and the
clipping are restated in numpy.  Pinned (tests/test_oracle_train.py) against the reference's own fixtures:
training-tiny logits and all 57 parameter gradients (TrainingGradientTests.cs:44-85), objective.json
(TrainingTests.cs:19-44) and the AdamW / cosine / clipping known answers (TrainingTests.cs:46-83).

Follows:
  * TrainableDecisionModel.Forward / EncoderLayerForward / HeadLayerForward (Laya.Training/TrainableDecisionModel.cs:248-468)
  * Ops.AttentionForward/ForwardUnit, Rotary, Dropout, Uniform, Mix (Laya.Training/Ops.cs:222-504)
  * RlcdObjective.Compute (Laya.Training/RlcdObjective.cs:57-155), Calibration.ProperReward (Laya/Runtime/Calibration.cs:76-119)
  * AdamW.Step, CosineSchedule, Gradients.ClipByGlobalNorm (Laya.Training/AdamW.cs:29-130)
"""
import math
from typing import Dict, List, Optional

import numpy as np
import torch
from torch.utils.checkpoint import checkpoint

from .model import EncoderConfig

M64 = (1 << 64) - 1


# ---------------------------------------------------------------------------------------------- dropout hash
def uniform(seed: int, index: np.ndarray) -> np.ndarray:
    """Ops.Uniform (Ops.cs:227-234): a counter-based uniform in [0, 1) per (seed, index), fp32."""
    idx = np.asarray(index, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & M64) + (idx + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return (z >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / (1 << 24))


def mix(seed: int, salt: int) -> int:
    """Ops.Mix (Ops.cs:236-241)."""
    z = (seed ^ ((salt * 0xD1B54A32D192ED03 + 0x8CB92BA72F3D8DD7) & M64)) & M64
    z = ((z ^ (z >> 33)) * 0xFF51AFD7ED558CCD) & M64
    return z ^ (z >> 33)


def salt(seed: int, layer: int, site: int) -> int:
    """TrainableDecisionModel.Salt (TrainableDecisionModel.cs:422)."""
    return mix(seed, layer * 16 + site + 1)


def dropout_mask(n: int, p: float, seed: int) -> np.ndarray:
    """Ops.Dropout's multiplier per flat index (Ops.cs:244-258): 0 where dropped, 1/(1-p) kept."""
    if p <= 0:
        return np.ones(n, np.float32)
    keep = np.float32(1.0) / (np.float32(1.0) - np.float32(p))
    return np.where(uniform(seed, np.arange(n, dtype=np.uint64)) < np.float32(p), np.float32(0), keep)


# ---------------------------------------------------------------------------------------------- torch model
def rope_tables(head_dim, theta, positions):
    half = head_dim // 2
    c = np.zeros((positions, half), np.float32)
    s = np.zeros((positions, half), np.float32)
    for i in range(half):
        inv = 1.0 / math.pow(theta, 2.0 * i / head_dim)
        for p_ in range(positions):
            c[p_, i] = np.float32(math.cos(p_ * inv))
            s[p_, i] = np.float32(math.sin(p_ * inv))
    return torch.from_numpy(c), torch.from_numpy(s)


def apply_rope(x, c, s):
    """Rotary.Apply (Ops.cs:490-503), rotate-half: x [L, heads, d]; c, s [L, d/2]."""
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    c = c[:, None, :]
    s = s[:, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


class TorchTrainModel:
    """fp32 autograd restatement of TrainableDecisionModel (concatenated segments, no padding)."""

    def __init__(self, cfg: EncoderConfig, weights: Dict[str, np.ndarray], head_dropout: float = 0.1):
        self.cfg = cfg
        self.p = {k: torch.tensor(np.asarray(v, np.float32), requires_grad=True) for k, v in weights.items()
                  if k != "temperature"}
        self.head_dropout = head_dropout
        self._rope = {}

    def rope(self, kind, L):
        theta = self.cfg.theta_global if kind == "global" else self.cfg.theta_local
        key = (kind, L)
        if key not in self._rope:
            self._rope[key] = rope_tables(self.cfg.head_dim, theta, max(L, 1))
        return self._rope[key]

    def ln(self, x, w, b, eps):
        mu = x.mean(-1, keepdim=True)
        var = ((x - mu) ** 2).mean(-1, keepdim=True)
        y = (x - mu) / torch.sqrt(var + eps) * self.p[w]
        return y + self.p[b] if (b and b in self.p) else y

    def lin(self, x, w, b=None):
        y = x @ self.p[w].t()
        return y + self.p[b] if (b and b in self.p) else y

    def attention(self, qkv, seg_start, seg_len, heads, window, kind=None, dropout=0.0, seed=0):
        """Ops.ForwardUnit (Ops.cs:329-366) over every (segment, head)."""
        H = qkv.shape[1] // 3
        d = H // heads
        scale = np.float32(1.0) / np.float32(math.sqrt(d))
        outs = []
        for s0, L in zip(seg_start, seg_len):
            x = qkv[s0:s0 + L]
            q = x[:, :H].reshape(L, heads, d)
            k = x[:, H:2 * H].reshape(L, heads, d)
            v = x[:, 2 * H:].reshape(L, heads, d)
            if kind is not None:
                c, s = self.rope(kind, L)
                q, k = apply_rope(q, c[:L], s[:L]), apply_rope(k, c[:L], s[:L])
            q, k = self.round_operand(q), self.round_operand(k)
            if L * L * heads > (1 << 27) and dropout == 0:
                # long rows (an 8192-token row holds 16 × 8192² scores): one head at a time, its scores recomputed
                # in the backward instead of kept, so the oracle stays within a few GB of host memory
                outs.append(torch.cat([checkpoint(self._head_unit, q[:, hh], k[:, hh], v[:, hh], window, float(scale),
                                                  use_reentrant=False) for hh in range(heads)], 1))
                continue
            sc = torch.einsum("thd,jhd->htj", q, k) * float(scale)
            if window >= 0:
                i = torch.arange(L)
                sc = sc.masked_fill((i[:, None] - i[None, :]).abs()[None] > window, float("-inf"))
            pr = torch.softmax(sc, -1)
            if dropout > 0:
                # Ops.DropoutIndex: (head << 42) | (row << 21) | key, with the segment's global row
                hh = np.arange(heads, dtype=np.uint64)[:, None, None]
                tt = (np.arange(L, dtype=np.uint64) + np.uint64(s0))[None, :, None]
                jj = np.arange(L, dtype=np.uint64)[None, None, :]
                idx = (hh << np.uint64(42)) | (tt << np.uint64(21)) | jj
                keep = np.float32(1) / (np.float32(1) - np.float32(dropout))
                m = np.where(uniform(seed, idx) < np.float32(dropout), np.float32(0), keep)
                pr = pr * torch.from_numpy(m)
            outs.append(torch.einsum("htj,jhd->thd", self.round_operand(pr), self.round_operand(v)).reshape(L, H))
        return torch.cat(outs, 0)

    def _head_unit(self, q, k, v, window, scale):
        """Ops.ForwardUnit (Ops.cs:329-366) for one (segment, head): q, k, v [L, d]."""
        L = q.shape[0]
        sc = (q @ k.t()) * scale
        if window >= 0:
            i = torch.arange(L)
            sc = sc.masked_fill((i[:, None] - i[None, :]).abs() > window, float("-inf"))
        return self.round_operand(torch.softmax(sc, -1)) @ self.round_operand(v)

    def forward(self, items, training=False, seed=0):
        """TrainableDecisionModel.Forward (TrainableDecisionModel.cs:248-353): option logits per item."""
        c = self.cfg
        seg_len = [len(it["ids"]) for it in items]
        seg_start = list(np.concatenate([[0], np.cumsum(seg_len)[:-1]]).astype(int))
        ids = torch.tensor(np.concatenate([np.asarray(it["ids"], np.int64) for it in items]))
        h = self.p["encoder.embeddings.tok_embeddings.weight"][ids]
        h = self.ln(h, "encoder.embeddings.norm.weight", "encoder.embeddings.norm.bias", c.norm_eps)
        for i in range(c.layers):
            lp = f"encoder.layers.{i}."
            normed = self.ln(h, lp + "attn_norm.weight", lp + "attn_norm.bias", c.norm_eps) \
                if (lp + "attn_norm.weight") in self.p else h
            qkv = self.lin(normed, lp + "attn.Wqkv.weight", lp + "attn.Wqkv.bias")
            kind = c.kind(i)
            att = self.attention(qkv, seg_start, seg_len, c.heads, c.half_window if kind == "sliding" else -1, kind)
            h = h + self.lin(att, lp + "attn.Wo.weight", lp + "attn.Wo.bias")
            normed = self.ln(h, lp + "mlp_norm.weight", lp + "mlp_norm.bias", c.norm_eps)
            wide = self.lin(normed, lp + "mlp.Wi.weight", lp + "mlp.Wi.bias")
            I = wide.shape[1] // 2
            act = torch.nn.functional.gelu(wide[:, :I]) * wide[:, I:]
            h = h + self.lin(act, lp + "mlp.Wo.weight", lp + "mlp.Wo.bias")
        h = self.ln(h, "encoder.final_norm.weight", "encoder.final_norm.bias", c.norm_eps)
        qt = torch.tensor(np.repeat([it["qtype"] for it in items], seg_len))
        h = h + self.p["type_emb.weight"][qt]
        T = h.shape[0]
        p_drop = self.head_dropout if training else 0.0
        heads = max(1, c.hidden // 64)
        for l in range(c.head_layers):
            lp = f"head.layers.{l}."
            normed = self.ln(h, lp + "norm1.weight", lp + "norm1.bias", 1e-5)
            qkv = self.lin(normed, lp + "self_attn.in_proj_weight", lp + "self_attn.in_proj_bias")
            ctx = self.attention(qkv, seg_start, seg_len, heads, -1, None, p_drop, salt(seed, l, 0))
            r = self.lin(ctx, lp + "self_attn.out_proj.weight", lp + "self_attn.out_proj.bias")
            r = r * torch.from_numpy(dropout_mask(r.numel(), p_drop, salt(seed, l, 1)).reshape(r.shape))
            h = h + r
            normed = self.ln(h, lp + "norm2.weight", lp + "norm2.bias", 1e-5)
            wide = self.lin(normed, lp + "linear1.weight", lp + "linear1.bias")
            dropped = torch.relu(wide) * torch.from_numpy(dropout_mask(wide.numel(), p_drop, salt(seed, l, 2)).reshape(wide.shape))
            out = self.lin(dropped, lp + "linear2.weight", lp + "linear2.bias")
            out = out * torch.from_numpy(dropout_mask(out.numel(), p_drop, salt(seed, l, 3)).reshape(out.shape))
            h = h + out
        rows = np.concatenate([np.asarray([s + max(0, m) for m in it["markers"]], np.int64)
                               for s, it in zip(seg_start, items)])
        x = self.ln(h[torch.tensor(rows)], "scorer.0.weight", "scorer.0.bias", 1e-5)
        y = torch.nn.functional.gelu(self.lin(x, "scorer.1.weight", "scorer.1.bias"))
        scores = self.lin(y, "scorer.3.weight", "scorer.3.bias")[:, 0]
        out, m = [], 0
        for it in items:
            k = len(it["markers"])
            out.append(scores[m:m + k])
            m += k
        return out

    def round_operand(self, x):
        """Operand rounding before a product: none in the fp32 reference path."""
        return x

    def grads(self):
        return {k: (v.grad.detach().numpy().copy() if v.grad is not None else np.zeros(v.shape, np.float32))
                for k, v in self.p.items()}

    def zero_grad(self):
        for v in self.p.values():
            v.grad = None


class TorchTrainModelBf16(TorchTrainModel):
    """The same model with bf16-operand products, the numerics torch.autocast(bfloat16) gives the reference notebook's
    DDP recipe: every product reads bf16-rounded operands and accumulates in fp32; the outputs that only feed another
    product (Wqkv / in_proj, Wi, head linear1) are stored in bf16; attention scores come from bf16 rotated q and k and
    the probabilities are rounded to bf16 before P·V."""

    BF16_OUTPUTS = ("attn.Wqkv.weight", "mlp.Wi.weight", "self_attn.in_proj_weight", "linear1.weight")

    def round_operand(self, x):
        return x.bfloat16().float()

    def lin(self, x, w, b=None):
        y = self.round_operand(x) @ self.round_operand(self.p[w]).t()
        if b and b in self.p:
            y = y + self.p[b]
        return self.round_operand(y) if w.endswith(self.BF16_OUTPUTS) else y


# ---------------------------------------------------------------------------------------------- objective
def proper_reward(q, target, qtype, w_sph=0.75, w_rps=1.0, log_floor=-9.21):
    """Calibration.ProperReward (Calibration.cs:76-119), all options unmasked."""
    q = np.asarray(q, np.float64)
    t = np.asarray(target, np.float64)
    log_score = float(np.sum(t * np.maximum(np.log(np.maximum(q, 1e-12)), log_floor)))
    reward = log_score + w_sph * (float(np.dot(t, q)) / max(math.sqrt(float(np.dot(q, q))), 1e-9))
    if qtype != 1:
        return reward
    k = max(len(q), 2)
    rps = float(np.sum((np.cumsum(q) - np.cumsum(t)) ** 2))
    return reward - w_rps * rps / (k - 1)


def softmax_f32(v):
    """SimdOps.Softmax (SimdOps.cs:275-291) in fp32."""
    v = np.asarray(v, np.float32)
    mx = np.max(v)
    e = np.exp((v - mx).astype(np.float32)).astype(np.float32)
    total = np.float32(0)
    for x in e:
        total = np.float32(total + x)
    return (e * (np.float32(1) / total if total > 0 else np.float32(0))).astype(np.float32)


def rlcd(logits: List[np.ndarray], targets: List[np.ndarray], qtypes: List[int], sigma: float, draws, scale=1.0,
         w_sph=0.75, w_rps=1.0, w_ce=1.0):
    """RlcdObjective.Compute with supplied draws (RlcdObjective.cs:57-155): (loss, policy, ce, mean reward, grads)."""
    n = len(logits)
    G = len(draws)
    eps = [[None] * n for _ in range(G)]
    reward = np.zeros((G, n))
    for g in range(G):
        for i in range(n):
            k = len(logits[i])
            e = np.asarray(draws[g][i][:k], np.float64) * sigma
            e = e - e.sum() / k
            eps[g][i] = e
            q = softmax_f32((np.asarray(logits[i], np.float64) + e).astype(np.float32))
            reward[g, i] = proper_reward(q, targets[i], qtypes[i], w_sph, w_rps)
    adv = reward - reward.mean(0, keepdims=True)
    count = G * n
    gm = adv.sum() / count
    std = math.sqrt(((adv - gm) ** 2).sum() / (count - 1)) if count > 1 else 0.0
    adv = adv / (std + 1e-6)
    policy = ce = 0.0
    grads = []
    s2 = sigma * sigma
    for i in range(n):
        k = len(logits[i])
        grad = np.zeros(k)
        for g in range(G):
            logp = -float(np.sum(eps[g][i] ** 2)) / (2 * s2)
            grad -= adv[g, i] * eps[g][i] / s2 / count
            policy -= adv[g, i] * logp / count
        p = softmax_f32(np.asarray(logits[i], np.float32)).astype(np.float64)
        t = np.asarray(targets[i], np.float64)
        ce -= float(np.sum(t * np.log(np.maximum(p, 1e-30)))) / n
        grad += w_ce * (p * t.sum() - t) / n
        grads.append((grad * scale).astype(np.float32))
    return policy + w_ce * ce, policy, ce, reward.sum() / count, grads


# ---------------------------------------------------------------------------------------------- optimizer
def adamw_step(data, grad, m, v, step, lr, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01):
    """AdamW.Step for one parameter (AdamW.cs:29-73), fp32 element arithmetic as the reference."""
    c1 = 1.0 - beta1 ** step
    c2 = 1.0 - beta2 ** step
    decay = np.float32(1.0 - lr * wd)
    step_size = np.float32(lr / c1)
    sqrt_c2 = np.float32(math.sqrt(c2))
    b1, b2, e = np.float32(beta1), np.float32(beta2), np.float32(eps)
    g = np.asarray(grad, np.float32)
    data *= decay
    m[:] = b1 * m + (np.float32(1) - b1) * g
    v[:] = b2 * v + (np.float32(1) - b2) * g * g
    data -= step_size * m / (np.sqrt(v) / sqrt_c2 + e)


def cosine_lr(base, step, total, minimum=1e-6):
    """CosineSchedule.At (AdamW.cs:93)."""
    return minimum + (base - minimum) * (1 + math.cos(math.pi * step / total)) / 2


def clip_by_global_norm(grads: List[np.ndarray], max_norm: float) -> float:
    """Gradients.ClipByGlobalNorm (AdamW.cs:103-130): returns the norm before clipping; scales in place."""
    norm = math.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in grads))
    coef = max_norm / (norm + 1e-6)
    if coef < 1.0:
        for g in grads:
            g *= np.float32(coef)
    return norm


# ---------------------------------------------------------------------------------------------- calibration
TYPE_NAMES = ("choice", "score", "noul")


def temperature_bucket(qtype: int, options: int) -> str:
    """QuestionTypes.TemperatureBucket (Base/Questions.cs:38-42)."""
    size = "2" if options <= 2 else "3-5" if options <= 5 else "6-10" if options <= 10 else "11+"
    return TYPE_NAMES[qtype if qtype in (0, 1) else 2] + ":" + size


def clamp_temperature(t: float, lo: float = 0.5, hi: float = 5.0) -> float:
    """Calibration.ClampTemperature (Laya/Runtime/Calibration.cs:23-24), in fp32."""
    t = np.float32(t)
    return float(np.clip(t, np.float32(lo), np.float32(hi))) if math.isfinite(t) else 1.0


def fit_one(samples) -> float:
    """TemperatureFitting.FitOne (TemperatureFitting.cs:36-72): golden-section search over log T of the mean soft
    cross-entropy, in double, samples in order; fewer than 10 samples give 1."""
    if len(samples) < 10:
        return 1.0

    def objective(log_t):
        t = math.exp(log_t)
        total = 0.0
        for _, logits, target in samples:
            z = [float(v) / t for v in logits]
            mx = -math.inf
            for v in z:
                mx = max(mx, v)
            s = 0.0
            for v in z:
                s += math.exp(v - mx)
            log_sum = mx + math.log(s)
            for v, tg in zip(z, target):
                total -= float(tg) * (v - log_sum)
        return total / len(samples)

    low, high = math.log(0.02), math.log(50)
    ratio = (math.sqrt(5) - 1) / 2
    a, b = high - ratio * (high - low), low + ratio * (high - low)
    fa, fb = objective(a), objective(b)
    it = 0
    while it < 80 and high - low > 1e-7:
        if fa < fb:
            high, b, fb = b, a, fa
            a = high - ratio * (high - low)
            fa = objective(a)
        else:
            low, a, fa = a, b, fb
            b = low + ratio * (high - low)
            fb = objective(b)
        it += 1
    return float(np.float32(math.exp((low + high) / 2)))


def fit_temperatures(samples, minimum_bucket_samples=30):
    """TemperatureFitting.Fit (TemperatureFitting.cs:78-101): samples are (qtype, logits, target); returns
    (by_type[3], {bucket: temperature} for buckets with enough samples, {bucket: count} in first-seen order)."""
    by_type = []
    for q in range(3):
        sel = [s for s in samples if s[0] == q]
        by_type.append(1.2 if not sel else clamp_temperature(fit_one(sel)))
    groups = {}
    for s in samples:
        groups.setdefault(temperature_bucket(s[0], len(s[1])), []).append(s)
    by_bucket = {k: clamp_temperature(fit_one(v)) for k, v in groups.items() if len(v) >= minimum_bucket_samples}
    return by_type, by_bucket, {k: len(v) for k, v in groups.items()}
