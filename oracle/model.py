"""Forward orchestration of the reference decision model, restated over the C oracle kernels.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows, in order:
  * ModernBertEncoder.Forward            (Laya/Models/ModernBertEncoder.cs:123-188)
  * DecisionModel.Forward / HeadForward  (Laya/Models/DecisionModel.cs:128-169, 236-307)
  * DecisionModel.ReadOut                (Laya/Models/DecisionModel.cs:171-229)
Weights are a dict of numpy arrays under the checkpoint's safetensors names.  A linear whose name is in
`q8` runs as a Q8_0 product (PackedMatrixQ8_0.Multiply, PackedMatrixQ8_0.cs:224-246): q8[name] = (q int8 [N, K],
d fp32 [N, K/32]).  Every other linear is the fp32 PackedMatrix product.
"""
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from . import (attention, dot, f32, gelu, geglu, layer_norm, linear_f32, q8_linear, relu, rope_table, softmax)


@dataclass
class EncoderConfig:
    """The ModernBertConfig fields the hot path reads (Laya/Models/ModernBertConfig.cs:60-117)."""
    hidden: int = 768
    intermediate: int = 1152
    layers: int = 22
    heads: int = 12
    vocab: int = 50368
    local_attention: int = 128
    global_every: int = 3
    layer_kinds: List[str] = field(default_factory=list)   # "global" | "sliding"; empty -> by global_every
    theta_global: float = 160000.0
    theta_local: float = 10000.0
    norm_eps: float = 1e-5
    head_layers: int = 2
    n_act: int = 2

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @property
    def half_window(self):
        """ModernBertConfig.SlidingHalfWindow (ModernBertConfig.cs:51): a token sees [i - w, i + w]."""
        return self.local_attention // 2

    def kind(self, i):
        if self.layer_kinds:
            return self.layer_kinds[i]
        return "global" if i % self.global_every == 0 else "sliding"

    @staticmethod
    def from_hf(cfg: dict, head_layers=2, n_act=2):
        kinds = [("global" if k == "full_attention" else "sliding") for k in cfg.get("layer_types", [])]
        rp = cfg.get("rope_parameters", {})
        tg = rp.get("full_attention", {}).get("rope_theta", cfg.get("global_rope_theta", 160000.0))
        tl = rp.get("sliding_attention", {}).get("rope_theta", cfg.get("local_rope_theta", 10000.0))
        return EncoderConfig(hidden=cfg["hidden_size"], intermediate=cfg["intermediate_size"],
                             layers=cfg["num_hidden_layers"], heads=cfg["num_attention_heads"],
                             vocab=cfg["vocab_size"], local_attention=cfg["local_attention"],
                             global_every=cfg.get("global_attn_every_n_layers", 3), layer_kinds=kinds,
                             theta_global=tg, theta_local=tl, norm_eps=cfg.get("norm_eps", 1e-5),
                             head_layers=head_layers, n_act=n_act)


def base_config():
    """ModernBERT-base geometry (config 1/2/3)."""
    return EncoderConfig()


def large_config():
    """ModernBERT-large geometry (config 4)."""
    return EncoderConfig(hidden=1024, intermediate=2624, layers=28, heads=16)


@dataclass
class Item:
    """DecisionModel.BatchItem (DecisionModel.cs:107): tokens, option-marker positions, question type."""
    ids: np.ndarray
    markers: List[int]
    qtype: int


class OracleModel:
    def __init__(self, cfg: EncoderConfig, weights: Dict[str, np.ndarray], q8: Optional[Dict] = None):
        self.cfg = cfg
        self.w = weights
        self.q8 = q8 or {}
        self._rope = {}

    def rope(self, kind, positions):
        theta = self.cfg.theta_global if kind == "global" else self.cfg.theta_local
        key = (kind, positions)
        if key not in self._rope:
            self._rope[key] = rope_table(self.cfg.head_dim, theta, positions)
        return self._rope[key]

    def linear(self, x, name, bias_name=None):
        b = self.w.get(bias_name) if bias_name else None
        if name in self.q8:
            q, d = self.q8[name]
            return q8_linear(x, q, d, b)
        return linear_f32(x, self.w[name], b)

    def ln(self, x, wname, bname, eps):
        return layer_norm(x, self.w[wname], self.w.get(bname) if bname else None, eps)

    # ModernBertEncoder.Forward (ModernBertEncoder.cs:123-188)
    def encoder(self, ids, seg_start, seg_len, record=None):
        c = self.cfg
        p = "encoder."
        if np.any((ids < 0) | (ids >= c.vocab)):
            raise ValueError("token id outside the vocabulary")
        h = f32(self.w[p + "embeddings.tok_embeddings.weight"][ids])
        h = self.ln(h, p + "embeddings.norm.weight", p + "embeddings.norm.bias", c.norm_eps)
        if record is not None:
            record["encoder.embeddings"] = h.copy()
        for i in range(c.layers):
            h = self.encoder_layer(h, i, seg_start, seg_len, record)
        h = self.ln(h, p + "final_norm.weight", p + "final_norm.bias", c.norm_eps)
        return h

    # One iteration of ModernBertEncoder.Forward's layer loop (ModernBertEncoder.cs:155-183)
    def encoder_layer(self, h, i, seg_start, seg_len, record=None):
        c = self.cfg
        lp = f"encoder.layers.{i}."
        maxlen = int(max(seg_len)) if len(seg_len) else 1
        if (lp + "attn_norm.weight") in self.w:
            normed = self.ln(h, lp + "attn_norm.weight", lp + "attn_norm.bias", c.norm_eps)
        else:
            normed = h.copy()          # layer 0: nn.Identity (ModernBertEncoder.cs:77-78, 161-164)
        qkv = self.linear(normed, lp + "attn.Wqkv.weight", lp + "attn.Wqkv.bias")
        kind = c.kind(i)
        window = c.half_window if kind == "sliding" else -1
        att = attention(qkv, c.hidden, c.heads, seg_start, seg_len, window, self.rope(kind, maxlen))
        h = h + self.linear(att, lp + "attn.Wo.weight", lp + "attn.Wo.bias")
        if record is not None:
            record[f"encoder.layers.{i}.attn_residual"] = h.copy()
        normed = self.ln(h, lp + "mlp_norm.weight", lp + "mlp_norm.bias", c.norm_eps)
        wide = self.linear(normed, lp + "mlp.Wi.weight", lp + "mlp.Wi.bias")
        act = geglu(wide)
        h = h + self.linear(act, lp + "mlp.Wo.weight", lp + "mlp.Wo.bias")
        if record is not None:
            record[f"encoder.layers.{i}.output"] = h.copy()
        return h

    # DecisionModel.HeadForward (DecisionModel.cs:236-307): nn.TransformerEncoderLayer(norm_first, ReLU)
    def head_layer(self, h, i, seg_start, seg_len):
        c = self.cfg
        lp = f"head.layers.{i}."
        heads = max(1, c.hidden // 64)
        normed = self.ln(h, lp + "norm1.weight", lp + "norm1.bias", 1e-5)
        qkv = self.linear(normed, lp + "self_attn.in_proj_weight", lp + "self_attn.in_proj_bias")
        ctx = attention(qkv, c.hidden, heads, seg_start, seg_len, -1, None)
        h = h + self.linear(ctx, lp + "self_attn.out_proj.weight", lp + "self_attn.out_proj.bias")
        normed = self.ln(h, lp + "norm2.weight", lp + "norm2.bias", 1e-5)
        wide = relu(self.linear(normed, lp + "linear1.weight", lp + "linear1.bias"))
        h = h + self.linear(wide, lp + "linear2.weight", lp + "linear2.bias")
        return h

    def states(self, items: List[Item], record=None):
        """Encoder + type embedding + head layers over the concatenated batch: [T, hidden]."""
        seg_len = np.array([len(it.ids) for it in items], np.int32)
        seg_start = np.concatenate([[0], np.cumsum(seg_len)[:-1]]).astype(np.int32)
        ids = np.concatenate([np.asarray(it.ids, np.int64) for it in items])
        h = self.encoder(ids, seg_start, seg_len, record)
        temb = self.w["type_emb.weight"]
        for i, it in enumerate(items):
            h[seg_start[i]:seg_start[i] + seg_len[i]] += temb[it.qtype]
        for i in range(self.cfg.head_layers):
            h = self.head_layer(h, i, seg_start, seg_len)
        return h, seg_start, seg_len

    # DecisionModel.ReadOut (DecisionModel.cs:171-229)
    def readout(self, item: Item, start: int, h):
        w = self.w
        H = self.cfg.hidden
        logits = np.zeros(len(item.markers), np.float32)
        for o, m in enumerate(item.markers):
            row = h[start + max(0, m)][None, :]
            x = layer_norm(row, w["scorer.0.weight"], w["scorer.0.bias"], 1e-5)[0]
            hid = np.array([dot(x, w["scorer.1.weight"][j]) + w["scorer.1.bias"][j] for j in range(H)],
                           np.float32)
            hid = gelu(hid)
            logits[o] = dot(hid, w["scorer.3.weight"][0]) + w["scorer.3.bias"][0]
        p = softmax(logits)
        k = np.float32(max(2, len(item.markers)))
        ent = np.float32(0)
        for v in p:
            ent -= v * np.float32(np.log(np.clip(v, np.float32(1e-9), np.float32(3.4e38)), dtype=np.float32))
        ent = np.float32(ent / np.float32(np.log(k, dtype=np.float32)))
        top1 = top2 = np.float32(0)
        for v in p:
            if v > top1:
                top2, top1 = top1, v
            elif v > top2:
                top2 = v
        act_in = np.concatenate([h[start], np.array([top1, top1 - top2, ent, k / np.float32(255)], np.float32)])
        a1 = np.array([dot(act_in, w["act_head.0.weight"][j]) + w["act_head.0.bias"][j]
                       for j in range(w["act_head.0.bias"].shape[0])], np.float32)
        a1 = gelu(a1)
        a2 = np.array([dot(a1, w["act_head.2.weight"][j]) + w["act_head.2.bias"][j]
                       for j in range(w["act_head.2.bias"].shape[0])], np.float32)
        return logits, softmax(a2), a2

    def forward(self, items: List[Item], record=None):
        """DecisionModel.Forward (DecisionModel.cs:128-169): per item (option logits, action probabilities)."""
        h, seg_start, _ = self.states(items, record)
        out = []
        for i, it in enumerate(items):
            logits, probs, _ = self.readout(it, int(seg_start[i]), h)
            out.append((logits, probs))
        return out
