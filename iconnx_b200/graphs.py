"""Synthetic ONNX-style graphs of the benchmark configurations, emitted
through the executor's builder API (add_input / add_initializer / add_node,
the reference's src/cuda/inference/mod.rs:306-347).

Every int8 Linear is the node sequence ONNX Runtime's dynamic quantisation
writes, which the engine's fusion pass turns into one kernel:

    DynamicQuantizeLinear(x) -> (q, s, z)
    MatMulInteger(q, W, z [, W_zp]) -> Cast(to=FLOAT) -> Mul(., Mul(s, W_scale))
    -> Add(., bias) [-> Div(sqrt2) -> Erf -> Add(1) -> Mul(x, .) -> Mul(0.5)]

Weights are seeded synthetic tensors (no checkpoint exists here):
W int8 uniform [-127, 127]; per-tensor W_scale 0.01 or per-column
U[0.005, 0.02] with W_zp int8 U[-8, 8]; biases and embedding / LayerNorm
weights N(0, 0.02).  Seed layout: x=0, W=1, bias=2, W2=3, w_scale=4, b_zp=5,
ids=6; layer l offsets seeds by 100*l.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import synth

SQRT2_F32 = np.float32(1.41421353816986083984375)


class _Namer:
    def __init__(self):
        self.k = 0

    def __call__(self, stem: str) -> str:
        self.k += 1
        return f"{stem}_{self.k}"


def dql(g, x: str, nm: _Namer):
    q, s, z = nm("q"), nm("s"), nm("z")
    g.add_node(nm("dql"), "DynamicQuantizeLinear", [x], [q, s, z])
    return q, s, z


def quant_linear(g, quantized, nm: _Namer, W: np.ndarray, w_scale: np.ndarray,
                 bias: np.ndarray | None, b_zp: np.ndarray | None = None, gelu: bool = False) -> str:
    """Emits the ORT dynamic-quantisation node chain for one Linear layer."""
    q, s, z = quantized
    wn, sn = nm("W"), nm("W_scale")
    g.add_initializer(wn, W)
    g.add_initializer(sn, w_scale.reshape(()) if w_scale.size == 1 else w_scale)
    ins = [q, wn, z]
    if b_zp is not None:
        zn = nm("W_zp")
        g.add_initializer(zn, b_zp)
        ins.append(zn)
    acc, cast, sc, o = nm("acc"), nm("cast"), nm("scale"), nm("deq")
    g.add_node(nm("mmi"), "MatMulInteger", ins, [acc])
    g.add_node(nm("cast"), "Cast", [acc], [cast], {"to": 1})
    g.add_node(nm("mul"), "Mul", [s, sn], [sc])
    g.add_node(nm("mul"), "Mul", [cast, sc], [o])
    if bias is not None:
        bn, ob = nm("bias"), nm("biased")
        g.add_initializer(bn, bias)
        g.add_node(nm("add"), "Add", [o, bn], [ob])
        o = ob
    if gelu:
        o = gelu_subgraph(g, o, nm)
    return o


def gelu_subgraph(g, x: str, nm: _Namer) -> str:
    """0.5 * x * (1 + erf(x / sqrt2)) as the exporter writes it."""
    c2, c1, ch = nm("sqrt2"), nm("one"), nm("half")
    g.add_initializer(c2, np.array(SQRT2_F32, np.float32))
    g.add_initializer(c1, np.array(1.0, np.float32))
    g.add_initializer(ch, np.array(0.5, np.float32))
    d, e, a, m, y = nm("div"), nm("erf"), nm("add1"), nm("mulx"), nm("gelu")
    g.add_node(nm("div"), "Div", [x, c2], [d])
    g.add_node(nm("erf"), "Erf", [d], [e])
    g.add_node(nm("add"), "Add", [e, c1], [a])
    g.add_node(nm("mul"), "Mul", [x, a], [m])
    g.add_node(nm("mul"), "Mul", [m, ch], [y])
    return y


# --------------------------------------------------------------- configs
def build_linear(g, M=128, K=768, N=768, batch_dim=True):
    """Config 1: one int8 Linear on x [1, 128, 768]."""
    nm = _Namer()
    shape = [1, M, K] if batch_dim else [M, K]
    g.add_input("x", shape)
    out = quant_linear(g, dql(g, "x", nm), nm, synth.int8_uniform((K, N), 1),
                       np.array([0.01], np.float32), synth.normal((N,), 0.02, 2))
    g.add_node("identity_out", "Identity", [out], ["y"])
    return "y"


def build_ffn(g, batch=32, seq=128, hidden=768, ffn=3072):
    """Config 2: int8 FFN block, x [batch*seq, hidden]."""
    nm = _Namer()
    g.add_input("x", [batch * seq, hidden])
    ws = np.array([0.01], np.float32)
    h = quant_linear(g, dql(g, "x", nm), nm, synth.int8_uniform((hidden, ffn), 1), ws,
                     synth.normal((ffn,), 0.02, 2), gelu=True)
    o = quant_linear(g, dql(g, h, nm), nm, synth.int8_uniform((ffn, hidden), 3), ws,
                     synth.normal((hidden,), 0.02, 102))
    g.add_node("identity_out", "Identity", [o], ["y"])
    return "y"


@dataclass
class BertConfig:
    layers: int = 6
    hidden: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 30522
    max_pos: int = 512
    per_channel: bool = False      # config 4: per-column w_scale and b_zp
    token_type: bool = False       # BERT adds a token-type embedding row
    eps: float = 1e-12
    # per-tensor weight scale (configs 3 / 4: 0.01; per-channel scales are
    # uniform in [w_scale / 2, 2 w_scale], i.e. [0.005, 0.02])
    w_scale: float = 0.01


DISTILBERT = BertConfig()

# With the configs' 0.01, int8 weights uniform over [-128, 127] act like
# weights of std ~0.74, so attention scores reach ~10^3 and softmax is nearly
# one-hot: any two fp32 evaluations of the scores (different summation
# orders) then differ by ~1 ulp of 10^3, which now and then moves a
# requantised attention output across a u8 boundary.  This scale gives an
# effective weight std of ~0.04 (trained BERT Linears; scores of order 1-10)
# for the strict whole-encoder parity checks.
REALISTIC_W_SCALE = 0.0005
BERT_BASE = BertConfig(layers=12, per_channel=True, token_type=True)


def build_bert(g, cfg: BertConfig, batch: int, seq: int) -> str:
    """Configs 3 / 4: DistilBERT-base / BERT-base encoder, int8 Linears,
    fp32 embeddings, LayerNorm and softmax attention.  Inputs input_ids and
    attention_mask (int64 [batch, seq]); output last_hidden_state."""
    nm = _Namer()
    H, nh = cfg.hidden, cfg.heads
    dh = H // nh
    g.add_input("input_ids", [batch, seq], np.int64)
    g.add_input("attention_mask", [batch, seq], np.int64)
    g.add_initializer("word_embeddings", synth.normal((cfg.vocab, H), 0.02, 7))
    g.add_initializer("position_embeddings", synth.normal((cfg.max_pos, H), 0.02, 8))
    g.add_initializer("position_ids", np.arange(seq, dtype=np.int64))
    g.add_node("emb_word", "Gather", ["word_embeddings", "input_ids"], ["we"])
    g.add_node("emb_pos", "Gather", ["position_embeddings", "position_ids"], ["pe"])
    g.add_node("emb_add", "Add", ["we", "pe"], ["emb"])
    x = "emb"
    if cfg.token_type:
        g.add_initializer("token_type_row", synth.normal((H,), 0.02, 9))
        g.add_node("emb_tt", "Add", [x, "token_type_row"], ["emb_tt"])
        x = "emb_tt"
    x = layernorm(g, x, nm, H, 10, cfg.eps)
    # additive attention mask [batch, 1, 1, seq]
    for name, v in (("mask_one", 1.0), ("mask_neg", -10000.0)):
        g.add_initializer(name, np.array(v, np.float32))
    g.add_node("mask_cast", "Cast", ["attention_mask"], ["mask_f"], {"to": 1})
    g.add_node("mask_inv", "Sub", ["mask_one", "mask_f"], ["mask_inv"])
    g.add_node("mask_scale", "Mul", ["mask_inv", "mask_neg"], ["mask_add"])
    g.add_node("mask_unsq", "Unsqueeze", ["mask_add"], ["mask_bias"], {"axes": [1, 2]})
    g.add_initializer("shape_heads", np.array([0, 0, nh, dh], np.int64))
    g.add_initializer("shape_hidden", np.array([0, 0, H], np.int64))
    g.add_initializer("attn_div", np.array(np.sqrt(dh), np.float32))

    for layer in range(cfg.layers):
        base = 100 * layer

        def lin(qz, K, N, seed, gelu=False):
            W = synth.int8_uniform((K, N), base + seed)
            if cfg.per_channel:
                ws = synth.uniform_f32((N,), 0.5 * cfg.w_scale, 2.0 * cfg.w_scale, base + seed + 40)
                bz = synth.int8_uniform((N,), base + seed + 50, -8, 8)
            else:
                ws, bz = np.array([cfg.w_scale], np.float32), None
            return quant_linear(g, qz, nm, W, ws, synth.normal((N,), 0.02, base + seed + 20), bz, gelu)

        qx = dql(g, x, nm)
        q = lin(qx, H, H, 11)
        k = lin(qx, H, H, 12)
        v = lin(qx, H, H, 13)

        def heads(t, perm):
            r, tr = nm("heads"), nm("heads_t")
            g.add_node(nm("reshape"), "Reshape", [t, "shape_heads"], [r])
            g.add_node(nm("transpose"), "Transpose", [r], [tr], {"perm": perm})
            return tr

        qh, kt, vh = heads(q, [0, 2, 1, 3]), heads(k, [0, 2, 3, 1]), heads(v, [0, 2, 1, 3])
        sc, sd, sm, p, ctx = nm("scores"), nm("scaled"), nm("masked"), nm("probs"), nm("ctx")
        g.add_node(nm("qk"), "MatMul", [qh, kt], [sc])
        g.add_node(nm("div"), "Div", [sc, "attn_div"], [sd])
        g.add_node(nm("add"), "Add", [sd, "mask_bias"], [sm])
        g.add_node(nm("softmax"), "Softmax", [sm], [p], {"axis": -1})
        g.add_node(nm("pv"), "MatMul", [p, vh], [ctx])
        ct, cr = nm("ctx_t"), nm("ctx_r")
        g.add_node(nm("transpose"), "Transpose", [ctx], [ct], {"perm": [0, 2, 1, 3]})
        g.add_node(nm("reshape"), "Reshape", [ct, "shape_hidden"], [cr])
        o = lin(dql(g, cr, nm), H, H, 14)
        r1 = nm("res")
        g.add_node(nm("add"), "Add", [o, x], [r1])
        x1 = layernorm(g, r1, nm, H, base + 15, cfg.eps)
        h = lin(dql(g, x1, nm), H, cfg.ffn, 16, gelu=True)
        o2 = lin(dql(g, h, nm), cfg.ffn, H, 17)
        r2 = nm("res")
        g.add_node(nm("add"), "Add", [o2, x1], [r2])
        x = layernorm(g, r2, nm, H, base + 18, cfg.eps)
    g.add_node("output", "Identity", [x], ["last_hidden_state"])
    return "last_hidden_state"


def build_attention(g, batch: int, seq: int, hidden: int = 768, heads: int = 12,
                    mask: str = "batch") -> str:
    """The encoder's self-attention block alone: graph inputs q, k, v
    [batch, seq, hidden] f32 and, for mask "batch" / "shared", an additive
    mask [batch, 1, 1, seq] / [1, 1, 1, seq]; Reshape / Transpose into heads,
    MatMul, Div(sqrt(dh)), Add(mask), Softmax, MatMul, Transpose, Reshape.
    Output "ctx" [batch, seq, hidden]."""
    nm = _Namer()
    dh = hidden // heads
    for t in ("q", "k", "v"):
        g.add_input(t, [batch, seq, hidden], np.float32)
    if mask == "batch":
        g.add_input("mask_bias", [batch, 1, 1, seq], np.float32)
    elif mask == "shared":
        g.add_input("mask_bias", [1, 1, 1, seq], np.float32)
    g.add_initializer("shape_heads", np.array([0, 0, heads, dh], np.int64))
    g.add_initializer("shape_hidden", np.array([0, 0, hidden], np.int64))
    g.add_initializer("attn_div", np.array(np.sqrt(dh), np.float32))

    def split(t, perm):
        r, tr = nm("heads"), nm("heads_t")
        g.add_node(nm("reshape"), "Reshape", [t, "shape_heads"], [r])
        g.add_node(nm("transpose"), "Transpose", [r], [tr], {"perm": perm})
        return tr

    qh, kt, vh = split("q", [0, 2, 1, 3]), split("k", [0, 2, 3, 1]), split("v", [0, 2, 1, 3])
    g.add_node("qk", "MatMul", [qh, kt], ["scores"])
    g.add_node("div", "Div", ["scores", "attn_div"], ["scaled"])
    sm_in = "scaled"
    if mask in ("batch", "shared"):
        g.add_node("add_mask", "Add", ["scaled", "mask_bias"], ["masked"])
        sm_in = "masked"
    g.add_node("softmax", "Softmax", [sm_in], ["probs"], {"axis": -1})
    g.add_node("pv", "MatMul", ["probs", vh], ["ctx_h"])
    g.add_node("ctx_t", "Transpose", ["ctx_h"], ["ctx_t"], {"perm": [0, 2, 1, 3]})
    g.add_node("ctx_r", "Reshape", ["ctx_t", "shape_hidden"], ["ctx"])
    return "ctx"


def attention_reference(q, k, v, heads: int, mask_bias=None) -> np.ndarray:
    """float64 evaluation of build_attention's graph (for tolerances)."""
    B, S, H = q.shape
    dh = H // heads

    def split(t):
        return t.astype(np.float64).reshape(B, S, heads, dh).transpose(0, 2, 1, 3)

    s = split(q) @ split(k).transpose(0, 1, 3, 2) / np.float64(np.float32(np.sqrt(dh)))
    if mask_bias is not None:
        s = s + mask_bias.astype(np.float64)
    s = np.exp(s - s.max(axis=-1, keepdims=True))
    p = s / s.sum(axis=-1, keepdims=True)
    return (p @ split(v)).transpose(0, 2, 1, 3).reshape(B, S, H)


def _u8(shape, seed, lo=0, hi=255):
    return synth.int8_uniform(shape, seed, lo - 128, hi - 128).view(np.uint8) ^ np.uint8(0x80)


def build_quantized_export(g, batch: int = 2, seq: int = 64, hidden: int = 768, ffn: int = 3072,
                           vocab: int = 1000, w_scale: float = REALISTIC_W_SCALE) -> tuple:
    """The layout of dynamically quantised transformer exports (the
    "_quantized" ONNX files of Transformers.js / Optimum): a u8 embedding
    table read with Gather and DequantizeLinear, and Linears whose u8 weights
    are stored transposed ("<name>_transposed_quantized" [N, K]) behind a
    runtime Transpose, with u8 weight zero points (scalar for the first
    Linear, per output column for the second).  Input input_ids [batch, seq];
    outputs (embedding f32, FFN1+GELU f32, FFN2 f32)."""
    nm = _Namer()
    g.add_input("input_ids", [batch, seq], np.int64)
    g.add_initializer("emb_quantized", _u8((vocab, hidden), 31))
    g.add_initializer("emb_scale", np.array(0.02, np.float32))
    g.add_initializer("emb_zero_point", np.array(128, np.uint8))
    g.add_node("emb_gather", "Gather", ["emb_quantized", "input_ids"], ["emb_q"])
    g.add_node("emb_dq", "DequantizeLinear", ["emb_q", "emb_scale", "emb_zero_point"], ["emb"])

    def linear(x, K, N, seed, per_col, gelu):
        wt = nm("W_transposed_quantized")
        g.add_initializer(wt, _u8((N, K), seed))
        w = nm("W")
        g.add_node(nm("transpose"), "Transpose", [wt], [w], {"perm": [1, 0]})
        sn, zn = nm("W_scale"), nm("W_zero_point")
        if per_col:
            g.add_initializer(sn, synth.uniform_f32((N,), 0.5 * w_scale, 2.0 * w_scale, seed + 1))
            g.add_initializer(zn, _u8((N,), seed + 2, 120, 136))
        else:
            g.add_initializer(sn, np.array(w_scale, np.float32))
            g.add_initializer(zn, np.array(131, np.uint8))
        q, s_, z = dql(g, x, nm)
        acc, cast, sc, o = nm("acc"), nm("cast"), nm("scale"), nm("deq")
        g.add_node(nm("mmi"), "MatMulInteger", [q, w, z, zn], [acc])
        g.add_node(nm("cast"), "Cast", [acc], [cast], {"to": 1})
        g.add_node(nm("mul"), "Mul", [s_, sn], [sc])
        g.add_node(nm("mul"), "Mul", [cast, sc], [o])
        bn, ob = nm("bias"), nm("biased")
        g.add_initializer(bn, synth.normal((N,), 0.02, seed + 3))
        g.add_node(nm("add"), "Add", [o, bn], [ob])
        return gelu_subgraph(g, ob, nm) if gelu else ob

    h = linear("emb", hidden, ffn, 40, False, True)
    y = linear(h, ffn, hidden, 50, True, False)
    g.add_node("out_h", "Identity", [h], ["ffn1"])
    g.add_node("out_y", "Identity", [y], ["ffn2"])
    return "emb", "ffn1", "ffn2"


def layernorm(g, x: str, nm: _Namer, H: int, seed: int, eps: float) -> str:
    gn, bn, y = nm("ln_gamma"), nm("ln_beta"), nm("ln")
    g.add_initializer(gn, (1.0 + synth.normal((H,), 0.02, seed + 1000)).astype(np.float32))
    g.add_initializer(bn, synth.normal((H,), 0.02, seed + 2000))
    g.add_node(nm("layernorm"), "LayerNormalization", [x, gn, bn], [y], {"axis": -1, "epsilon": eps})
    return y


def bert_inputs(batch: int, seq: int, vocab: int = 30522, seed: int = 6):
    return {"input_ids": synth.token_ids((batch, seq), seed, vocab),
            "attention_mask": np.ones((batch, seq), np.int64)}


def gemm_ops_per_sequence(cfg: BertConfig, seq: int) -> float:
    """int8 GEMM work (2*M*N*K) of one sequence through the encoder."""
    H, F = cfg.hidden, cfg.ffn
    return cfg.layers * 2.0 * seq * (4 * H * H + 2 * H * F)
