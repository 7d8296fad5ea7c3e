"""Oracle of the Mica decoder: the reference's Qwen3.5 forward restated for the CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the parity tests and bench.py's CPU arms use it as the checker;
the product never imports it.  Pinned (tests/test_oracle_decoder.py) against the reference's qwen35-tiny fixture:
every layer's mixer output and output, the final norm and the last position's logits, both in fp32
(reference.safetensors, Qwen35ParityTests.cs:45-86) and with every product in Q8_0 as ggml computes it
(reference-q8_0.safetensors, Qwen35ParityTests.cs:95-136).

Follows Qwen35Model (Mica/Models/Qwen35Model.cs):
  * Forward (:462-532): embeddings, layers (mixer then MLP), final RMSNorm of every row (recorded) and of the last;
  * FullAttention (:628-731): RMSNorm → qkv (q | gate interleaved per head, then k, v) → per-head RMSNorm of q and k,
    rotate-half RoPE on the first rotary_dim dimensions (inv_freq in fp32, angle = pos · inv_freq in fp32) → causal
    GQA softmax attention → · sigmoid(gate) → o_proj → residual;
  * LinearAttention (:784-921): RMSNorm → in_proj [qkv conv channels | z | b | a] → causal depthwise conv (kernel 4,
    separate multiply and add per tap, zero history) → SiLU → L2 norm of q (· 1/sqrt(dk)) and k per key head →
    β = sigmoid(b), g = exp(−exp(A_log) · softplus(a + dt_bias)) (subnormal → 0) → the gated delta rule per value head
    (Recurrence :924-972, C: lo_delta_rule) → RMSNormGated(o, z) → out_proj → residual;
  * Mlp (:602-621): RMSNorm → [gate; up] → silu(gate) · up → down → residual;
  * Logits (:563-575) / TokenTable.QuantizedLogits (:1091-1111): the tied embedding's rows for the requested ids;
  * DecoderKernels (Base/Numerics/DecoderKernels.cs) for RMSNorm, L2Normalize, RmsNormGated, SiLU, sigmoid, softplus.
With precision "q8_0" every projection and the token table are ggml Q8_0 (weights quantized at load from their bf16
values, activations quantized at every product) as `Qwen35Model(..., WeightPrecision.Q8_0)` runs them.
"""
import json
import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np

from . import f32, lib, q8_linear, q8_quantize_weights, q8_quantize_activations


@dataclass
class DecoderConfig:
    """Qwen35Config (Mica/Models/Qwen35Config.cs:60-130)."""
    hidden: int
    intermediate: int
    layers: int
    vocab: int
    eps: float
    kinds: List[str]               # "linear" | "full"
    heads: int
    kv_heads: int
    head_dim: int
    rope_theta: float
    partial_rotary: float
    lin_k_heads: int
    lin_v_heads: int
    lin_dk: int
    lin_dv: int
    conv_kernel: int

    @property
    def rotary_dim(self):
        return int(self.head_dim * self.partial_rotary)

    @property
    def key_dim(self):
        return self.lin_k_heads * self.lin_dk

    @property
    def value_dim(self):
        return self.lin_v_heads * self.lin_dv

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    @staticmethod
    def from_hf(cfg: dict):
        t = cfg.get("text_config", cfg)
        rope = t.get("rope_parameters", {})
        kinds = [("full" if k == "full_attention" else "linear") for k in t["layer_types"]]
        return DecoderConfig(hidden=t["hidden_size"], intermediate=t["intermediate_size"], layers=t["num_hidden_layers"],
                             vocab=t["vocab_size"], eps=float(t.get("rms_norm_eps", 1e-6)), kinds=kinds,
                             heads=t["num_attention_heads"], kv_heads=t["num_key_value_heads"],
                             head_dim=t.get("head_dim", t["hidden_size"] // t["num_attention_heads"]),
                             rope_theta=float(rope.get("rope_theta", 1e7)),
                             partial_rotary=float(rope.get("partial_rotary_factor", 0.25)),
                             lin_k_heads=t["linear_num_key_heads"], lin_v_heads=t["linear_num_value_heads"],
                             lin_dk=t["linear_key_head_dim"], lin_dv=t["linear_value_head_dim"],
                             conv_kernel=t["linear_conv_kernel_dim"])


def mica_config():
    """Config 5's geometry: 32 layers of [DeltaNet ×3, full ×1], h 2560, SwiGLU 9216, vocab 151936, DeltaNet 16 key and
    16 value heads × 128 (ratio 1), full attention 16 q / 4 kv heads × 128, RoPE θ 1e7 on a quarter of each head."""
    return DecoderConfig(hidden=2560, intermediate=9216, layers=32, vocab=151936, eps=1e-6,
                         kinds=(["linear"] * 3 + ["full"]) * 8, heads=16, kv_heads=4, head_dim=128, rope_theta=1e7,
                         partial_rotary=0.25, lin_k_heads=16, lin_v_heads=16, lin_dk=128, lin_dv=128, conv_kernel=4)


def _softplus(x):
    """DecoderKernels.Softplus (DecoderKernels.cs:154): x > 20 ? x : (float)log(1 + exp(x)) in double."""
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def _sigmoid_scalar(x):
    """DecoderKernels.Sigmoid(float) (DecoderKernels.cs:152): 1 / (1 + MathF.Exp(-x))."""
    x = np.asarray(x, np.float32)
    return (np.float32(1) / (np.float32(1) + np.exp(-x))).astype(np.float32)


class OracleState:
    """Qwen35State (Qwen35Model.cs:38-197): what the decoder remembers of the tokens it has read — keys and values of
    every full-attention layer (normed and rotated, fp32), the conv tail (the last kernel − 1 pre-convolution rows)
    and the delta-rule state [value heads, dk, dv] of every DeltaNet layer, and the token count."""

    def __init__(self, cfg: "DecoderConfig"):
        self.length = 0
        self.keys, self.values, self.tail, self.rec = {}, {}, {}, {}
        for i, kind in enumerate(cfg.kinds):
            if kind == "full":
                self.keys[i] = np.zeros((0, cfg.kv_heads, cfg.head_dim), np.float32)
                self.values[i] = np.zeros((0, cfg.kv_heads, cfg.head_dim), np.float32)
            else:
                self.tail[i] = np.zeros((cfg.conv_kernel - 1, cfg.conv_dim), np.float32)
                self.rec[i] = np.zeros((cfg.lin_v_heads, cfg.lin_dk, cfg.lin_dv), np.float32)

    def clone(self):
        """Clone (:112-117): an independent copy."""
        o = OracleState.__new__(OracleState)
        o.length = self.length
        o.keys = {i: a.copy() for i, a in self.keys.items()}
        o.values = {i: a.copy() for i, a in self.values.items()}
        o.tail = {i: a.copy() for i, a in self.tail.items()}
        o.rec = {i: a.copy() for i, a in self.rec.items()}
        return o

    def save(self):
        """Save (:127-131): the length and copies of the conv tails and recurrent states (keys and values stay)."""
        return (self.length, {i: a.copy() for i, a in self.tail.items()}, {i: a.copy() for i, a in self.rec.items()})

    def rewind(self, mark):
        """Rewind (:134-143): back to a saved point of this state; a mark cannot advance it."""
        length, tail, rec = mark
        if length > self.length:
            raise ValueError("a mark can only rewind, not advance")
        for i in self.tail:
            self.tail[i] = tail[i].copy()
            self.rec[i] = rec[i].copy()
        for i in self.keys:
            self.keys[i] = self.keys[i][:length].copy()
            self.values[i] = self.values[i][:length].copy()
        self.length = length


class OracleDecoder:
    """Qwen35Model forward over one sequence (fp32 or Q8_0 products), from an empty state or continuing one."""

    def __init__(self, cfg: DecoderConfig, weights: Dict[str, np.ndarray], precision: str = "f32",
                 q8: Optional[Dict[str, tuple]] = None, prefix: str = "model."):
        self.cfg = cfg
        self.precision = precision
        self.w = {k: np.asarray(v, np.float32) for k, v in weights.items()}
        self.p = prefix
        self.q8 = dict(q8 or {})
        L = lib()
        self.L = L
        # inv_freq = 1 / theta^(2i / rotary_dim) in fp32 (Qwen35Model.cs:247-253)
        half = cfg.rotary_dim // 2
        self.inv_freq = np.array([np.float32(1) / np.power(np.float32(cfg.rope_theta), np.float32(2 * i) /
                                                           np.float32(cfg.rotary_dim), dtype=np.float32)
                                  for i in range(half)], np.float32)

    # ---------------------------------------------------------------------------------------------- pieces
    def W(self, name):
        return self.w[self.p + name]

    def one_plus(self, name):
        return (np.float32(1) + self.W(name)).astype(np.float32)

    def rms(self, x, name=None, scale=None):
        x = f32(x)
        rows, n = x.shape
        out = np.empty_like(x)
        sc = f32(self.one_plus(name) if scale is None else scale)
        self.L.lo_rms_norm_rows(x, rows, n, sc, np.float32(self.cfg.eps), out)
        return out

    def proj(self, x, names: List[str]):
        """Stack (Qwen35Model.cs:300-345): sibling projections stacked along the output, one product."""
        if self.precision == "q8_0":
            key = "|".join(names)
            if key not in self.q8:
                self.q8[key] = q8_quantize_weights(np.concatenate([self.W(n) for n in names], 0))
            qw, dw = self.q8[key]
            return q8_linear(f32(x), qw, dw)
        from . import linear_f32
        return linear_f32(f32(x), f32(np.concatenate([self.W(n) for n in names], 0)))

    def embed(self, ids):
        if self.precision == "q8_0":
            if "embed" not in self.q8:
                self.q8["embed"] = q8_quantize_weights(self.W("embed_tokens.weight"))
            q, d = self.q8["embed"]
            # TokenTable.Row (Qwen35Model.cs:1076-1082): q · scale, per 32-block
            return (q[ids].astype(np.float32) * np.repeat(d[ids], 32, axis=1)).astype(np.float32)
        return self.W("embed_tokens.weight")[ids].copy()

    def logits(self, hidden, ids):
        """Logits (Qwen35Model.cs:563-575) or QuantizedLogits (:1091-1111) for the given ids."""
        h = f32(hidden).reshape(1, -1)
        if self.precision == "q8_0":
            if "embed" not in self.q8:
                self.q8["embed"] = q8_quantize_weights(self.W("embed_tokens.weight"))
            q, d = self.q8["embed"]
            return q8_linear(h, q[ids], d[ids])[0]
        from . import dot
        table = self.W("embed_tokens.weight")
        return np.array([dot(h[0], table[i]) for i in ids], np.float32)

    # ---------------------------------------------------------------------------------------------- layers
    def full_attention(self, i, x, state=None, checkpoints=(), snapshots=()):
        """Each row's key and value join the state's cache (positions continue from its length); every row attends
        to the cache up to itself.  Snapshots take the keys and values up to their checkpoint (:734-749)."""
        c = self.cfg
        p = f"layers.{i}.self_attn."
        T = x.shape[0]
        hd, H, KV = c.head_dim, c.heads, c.kv_heads
        normed = self.rms(x, f"layers.{i}.input_layernorm.weight")
        qkv = self.proj(normed, [p + "q_proj.weight", p + "k_proj.weight", p + "v_proj.weight"])
        qw = 2 * H * hd
        kvw = KV * hd
        half = c.rotary_dim // 2
        qn, kn = self.one_plus(p + "q_norm.weight"), self.one_plus(p + "k_norm.weight")
        start = state.length if state is not None else 0
        pos = np.arange(start, start + T, dtype=np.float32)
        ang = (pos[:, None] * self.inv_freq[None, :]).astype(np.float32)
        cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        q = np.empty((T, H, hd), np.float32)
        g = np.empty((T, H, hd), np.float32)
        for h in range(H):
            q[:, h] = self.rms(qkv[:, h * 2 * hd:h * 2 * hd + hd], scale=qn)
            g[:, h] = qkv[:, h * 2 * hd + hd:(h + 1) * 2 * hd]
        k = np.stack([self.rms(qkv[:, qw + h * hd:qw + (h + 1) * hd], scale=kn) for h in range(KV)], 1)
        v = np.stack([qkv[:, qw + kvw + h * hd:qw + kvw + (h + 1) * hd] for h in range(KV)], 1)
        for arr in (q, k):
            a, b = arr[..., :half].copy(), arr[..., half:2 * half].copy()
            arr[..., :half] = a * cos[:, None, :] - b * sin[:, None, :]
            arr[..., half:2 * half] = b * cos[:, None, :] + a * sin[:, None, :]
        if state is not None:
            k = np.concatenate([state.keys[i][:start], k], 0)
            v = np.concatenate([state.values[i][:start], v], 0)
            state.keys[i], state.values[i] = k, v
            for cp, snap in zip(checkpoints, snapshots):
                snap.keys[i], snap.values[i] = k[:start + cp].copy(), v[:start + cp].copy()
        scale = np.float32(1) / np.float32(math.sqrt(hd))
        out = np.zeros((T, H, hd), np.float32)
        groups = H // KV
        from . import dot
        for h in range(H):
            kh = h // groups
            for t in range(T):
                at = start + t
                s = np.array([dot(q[t, h], k[j, kh]) for j in range(at + 1)], np.float32) * scale
                e = np.exp(s - s.max()).astype(np.float32)
                tot = np.float32(0)
                for val in e:
                    tot = np.float32(tot + val)
                inv = np.float32(1) / tot
                o = np.zeros(hd, np.float32)
                for j in range(at + 1):
                    o = (np.float64(e[j] * inv) * v[j, kh].astype(np.float64) + o).astype(np.float32)
                out[t, h] = o
        out = out.reshape(T, H * hd)
        self.L.lo_multiply_sigmoid(out.reshape(-1), f32(g.reshape(T, H * hd)).reshape(-1), out.size)
        return self.proj(out, [p + "o_proj.weight"])

    def linear_attention(self, i, x, state=None, checkpoints=(), snapshots=()):
        """The conv reads the state's tail before the rows and the recurrence continues its state; both are advanced.
        A checkpoint splits the recurrence there and copies the tail and the state out (:814-830, :880-895)."""
        c = self.cfg
        p = f"layers.{i}.linear_attn."
        T = x.shape[0]
        cd, kd, vd = c.conv_dim, c.key_dim, c.value_dim
        VH, KH, dk, dv = c.lin_v_heads, c.lin_k_heads, c.lin_dk, c.lin_dv
        normed = self.rms(x, f"layers.{i}.input_layernorm.weight")
        proj = self.proj(normed, [p + "in_proj_qkv.weight", p + "in_proj_z.weight", p + "in_proj_b.weight",
                                  p + "in_proj_a.weight"])
        wconv = self.W(p + "conv1d.weight").reshape(cd, c.conv_kernel)     # [channel, tap]
        K = c.conv_kernel
        prev = state.tail[i] if state is not None else np.zeros((K - 1, cd), np.float32)
        hist = np.concatenate([prev, proj[:, :cd]], 0)
        if state is not None:
            for cp, snap in zip(checkpoints, snapshots):
                snap.tail[i] = hist[cp:cp + K - 1].copy()
            state.tail[i] = hist[T:T + K - 1].copy()
        conv = np.zeros((T, cd), np.float32)
        for j in range(K):                                                   # taps in order, multiply then add
            conv = (conv + (wconv[:, j][None, :] * hist[j:j + T])).astype(np.float32)
        conv = f32(conv)
        self.L.lo_silu_vec(conv.reshape(-1), conv.size)
        qscale = np.float32(1) / np.float32(math.sqrt(dk))
        for t in range(T):
            for h in range(KH):
                qv = np.ascontiguousarray(conv[t, h * dk:(h + 1) * dk])
                self.L.lo_l2_normalize(qv, dk, np.float32(1e-6), qscale)
                conv[t, h * dk:(h + 1) * dk] = qv
                kv = np.ascontiguousarray(conv[t, kd + h * dk:kd + (h + 1) * dk])
                self.L.lo_l2_normalize(kv, dk, np.float32(1e-6), np.float32(1))
                conv[t, kd + h * dk:kd + (h + 1) * dk] = kv
        b = proj[:, cd + vd:cd + vd + VH]
        a = proj[:, cd + vd + VH:cd + vd + 2 * VH]
        beta = _sigmoid_scalar(b)
        nega = (-np.exp(self.W(p + "A_log").astype(np.float32))).astype(np.float32)
        g = np.exp((nega[None, :] * _softplus(a + self.W(p + "dt_bias")[None, :])).astype(np.float32)).astype(np.float32)
        g = np.where(np.abs(g) < np.finfo(np.float32).tiny, np.float32(0), g).astype(np.float32)
        core = np.zeros((T, vd), np.float32)
        ratio = VH // KH
        flat = conv.reshape(-1)
        beta = f32(beta)
        g = f32(g)
        gf, bf = g.reshape(-1), beta.reshape(-1)
        for h in range(VH):
            kh = h // ratio
            S = state.rec[i][h].copy() if state is not None else np.zeros((dk, dv), np.float32)
            tmp = np.zeros(T * vd, np.float32)
            done = 0
            for until, snap in list(zip(checkpoints, snapshots)) + [(T, None)]:
                if until > done:
                    o0 = done * cd
                    seg = np.zeros((until - done) * vd, np.float32)
                    self.L.lo_delta_rule(S, dk, dv, until - done, f32(flat[o0 + kh * dk:]), f32(flat[o0 + kd + kh * dk:]),
                                         f32(flat[o0 + 2 * kd + h * dv:]), cd, f32(gf[done * VH + h:]),
                                         f32(bf[done * VH + h:]), VH, seg, vd)
                    tmp[done * vd:until * vd] = seg
                    done = until
                if snap is not None:
                    snap.rec[i][h] = S
            if state is not None:
                state.rec[i][h] = S
            core[:, h * dv:(h + 1) * dv] = tmp.reshape(T, vd)[:, :dv]
        z = proj[:, cd:cd + vd]
        wn = self.W(p + "norm.weight")
        for t in range(T):
            for h in range(VH):
                o = f32(core[t, h * dv:(h + 1) * dv])
                res = np.empty(dv, np.float32)
                self.L.lo_rms_norm_gated(o, f32(z[t, h * dv:(h + 1) * dv]), f32(wn), dv, np.float32(c.eps), res)
                core[t, h * dv:(h + 1) * dv] = res
        return self.proj(core, [p + "out_proj.weight"])

    def mlp(self, i, x):
        normed = self.rms(x, f"layers.{i}.post_attention_layernorm.weight")
        gu = self.proj(normed, [f"layers.{i}.mlp.gate_proj.weight", f"layers.{i}.mlp.up_proj.weight"])
        T, I = x.shape[0], self.cfg.intermediate
        act = np.empty((T, I), np.float32)
        self.L.lo_silu_multiply(f32(gu), T, I, act)
        return self.proj(act, [f"layers.{i}.mlp.down_proj.weight"])

    def layer(self, i, x, state=None, checkpoints=(), snapshots=()):
        """One decoder layer: (mixer output, layer output) — Forward's loop body (Qwen35Model.cs:485-500)."""
        mix = self.full_attention if self.cfg.kinds[i] == "full" else self.linear_attention
        mixer = mix(i, x, state, checkpoints, snapshots)
        x = (x + mixer).astype(np.float32)
        x = (x + self.mlp(i, x)).astype(np.float32)
        return mixer, x

    def new_state(self):
        """NewState (Qwen35Model.cs:419): a state that has read nothing."""
        return OracleState(self.cfg)

    def forward(self, ids, record: bool = True, state: Optional[OracleState] = None, checkpoints=()):
        """Returns (states by the reference's recorder names, the final-normed last hidden state).  With `state`, the
        tokens are read after what it holds and it is advanced; `checkpoints` (token counts 1..len(ids), ascending)
        add a third result, one new state per checkpoint (Qwen35Sequence.Checkpoints / Snapshots, :214-221)."""
        ids = np.asarray(ids, np.int64)
        if checkpoints and state is None:
            state = self.new_state()
        snapshots = [self.new_state() for _ in checkpoints]
        start = state.length if state is not None else 0
        x = self.embed(ids)
        states = {"embeddings": x.copy()} if record else {}
        for i in range(self.cfg.layers):
            mixer, x = self.layer(i, x, state, tuple(checkpoints), snapshots)
            if record:
                states[f"layers.{i}.mixer"] = mixer
                states[f"layers.{i}"] = x.copy()
        if state is not None:
            state.length = start + len(ids)
            for cp, snap in zip(checkpoints, snapshots):
                snap.length = start + cp
        normed = self.rms(x, "norm.weight")
        if record:
            states["norm"] = normed
        if checkpoints:
            return states, normed[-1].copy(), snapshots
        return states, normed[-1].copy()


def load_tiny(golden_dir):
    """The reference's qwen35-tiny fixture (tests/golden/qwen35_tiny*.npz, made by make_golden.py)."""
    import os
    g = json.load(open(os.path.join(golden_dir, "qwen35_tiny.json")))
    cfg = DecoderConfig.from_hf(g["config"])
    w = dict(np.load(os.path.join(golden_dir, "qwen35_tiny_model.npz")))
    ref = dict(np.load(os.path.join(golden_dir, "qwen35_tiny_reference.npz")))
    refq = dict(np.load(os.path.join(golden_dir, "qwen35_tiny_reference_q8_0.npz")))
    return cfg, w, np.asarray(g["input_ids"], np.int64), ref, refq
