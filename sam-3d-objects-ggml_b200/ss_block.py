"""One sparse-structure flow DiT block on the device (the shape group of
cpp_ggml/src/ss_flow_graph.cpp:180-388), built from libb2q's entry points:

    h = modulate(norm(x), scale_msa, shift_msa)          b2q_norm_modulate_q8
    qkv = h . W_qkv + b_qkv                               b2q_mul_mat_prepared
    q, k = rms_norm_head(q) * gq, rms_norm_head(k) * gk   b2q_qkv_heads (fp16 q, k, v)
    o = softmax(q k^T / sqrt(D)) v                        attention core (see below), Q8_0 out
    x = x + gate_msa * (o . W_out + b_out)               _gate_residual
    h = norm(x) * w2 + b2n                                b2q_layer_norm_q8           (cross-attention,
    q = h . W_xq + b_xq;  k | v = cond . W_xkv + b_xkv    b2q_mul_mat_prepared         :308-352)
    o = softmax(q k^T / sqrt(D)) v                        b2q_rows_to_heads, attention core
    x = x + (o . W_xout + b_xout)                         _gate_residual
    h = modulate(norm(x), scale_mlp, shift_mlp)          b2q_norm_modulate_q8
    x = x + gate_mlp * (gelu(h . W1 + b1) . W2 + b2)     _gelu_q8 + _gate_residual

Every linear, norm, quantize, epilogue and attention core is libb2q's (the
attention: b2q_attention_f16_q8, tensor cores, fp16 q, k, v and o, fp32 softmax,
its fp16 output quantized in the same kernel into the to_out linear's Q8_0
activations -- the bytes of b2q_heads_act_prepare of b2q_attention_f16's rows).
Modulation vectors are shared by
the batch (the CFG branches of one step share the timestep embedding).  The
4-token pose group (whose tiny linears run on the few-token kernel) and the
adaLN projection are not part of this step.
"""
from __future__ import annotations

import b2q


class SsBlock:
    """Packed weights of one block and its forward pass on fp32 [B*T, C] x."""

    # (out, in) of each linear for width C and hidden width Hd
    @staticmethod
    def shapes(C: int, hidden: int) -> dict:
        return {"qkv": (3 * C, C), "out": (C, C), "xq": (C, C), "xkv": (2 * C, C), "xout": (C, C),
                "fc1": (hidden, C), "fc2": (C, hidden)}

    def __init__(self, dev, weights: dict, C: int = 1024, heads: int = 16, mlp_ratio: int = 4,
                 wtype: int = b2q.TYPE_Q8_0, seed: int = 0):
        """weights: GGUF rows (uint8 numpy [out, row bytes]) of every linear in
        shapes(); the biases, gammas, norm2 affine and modulation vectors are seeded."""
        import numpy as np
        import torch
        self.C, self.H, self.D, self.hidden = C, heads, C // heads, C * mlp_ratio
        self.wtype = wtype
        rng = np.random.default_rng(seed)
        self.raw = {}
        self.packed = {}
        for name, (n, k) in self.shapes(C, self.hidden).items():
            w = weights[name]
            assert w.shape[0] == n
            self.raw[name] = w
            self.packed[name] = b2q.weight_pack(wtype, torch.from_numpy(w).to(dev), k)
        f = lambda n, s=1.0: torch.from_numpy((rng.standard_normal(n) * s).astype(np.float32)).to(dev)  # noqa: E731
        self.vec = {"b_qkv": f(3 * C, 0.1), "b_out": f(C, 0.1), "b1": f(self.hidden, 0.1), "b2": f(C, 0.1),
                    "gq": 1.0 + f(C, 0.1), "gk": 1.0 + f(C, 0.1),
                    "shift_msa": f(C, 0.1), "scale_msa": f(C, 0.1), "gate_msa": f(C, 0.5),
                    "shift_mlp": f(C, 0.1), "scale_mlp": f(C, 0.1), "gate_mlp": f(C, 0.5),
                    "n2w": 1.0 + f(C, 0.1), "n2b": f(C, 0.1), "b_xq": f(C, 0.1), "b_xkv": f(2 * C, 0.1),
                    "b_xout": f(C, 0.1)}
        self.dev = dev

    def forward(self, x, B: int, T: int, cond, n_cond: int, stream=None):
        """x: fp32 [B*T, C] residual stream, updated in place and returned;
        cond: fp32 [B*n_cond, C] condition tokens."""
        C, H, D, v = self.C, self.H, self.D, self.vec

        def attend(q, k, vv):  # -> the to_out linear's Q8_0 prepared activations
            return b2q.attention_f16_q8(q, k, vv, stream=stream)

        M = B * T
        act = b2q.norm_modulate_q8(x, 1e-6, v["scale_msa"], v["shift_msa"], stream=stream)
        qkv = b2q.mul_mat_prepared(self.packed["qkv"], 3 * C, C, act, M, bias=v["b_qkv"], stream=stream)
        q, k, vv = b2q.qkv_heads(qkv, B, T, H, D, v["gq"], v["gk"], 1e-6, stream=stream)
        act_o = attend(q, k, vv)
        b2q.mul_mat_prepared_gate_residual(self.packed["out"], C, C, act_o, M, x, bias=v["b_out"],
                                           gate=v["gate_msa"], out=x, stream=stream)
        # cross-attention to the condition tokens
        act = b2q.layer_norm_q8(x, 1e-6, v["n2w"], v["n2b"], stream=stream)
        xq = b2q.mul_mat_prepared(self.packed["xq"], C, C, act, M, bias=v["b_xq"], stream=stream)
        act_c = b2q.act_prepare(cond, stream=stream)
        xkv = b2q.mul_mat_prepared(self.packed["xkv"], 2 * C, C, act_c, B * n_cond, bias=v["b_xkv"], stream=stream)
        (q,) = b2q.rows_to_heads(xq, B, T, H, D, 1, stream=stream)
        k, vv = b2q.rows_to_heads(xkv, B, n_cond, H, D, 2, stream=stream)
        act_o = attend(q, k, vv)
        b2q.mul_mat_prepared_gate_residual(self.packed["xout"], C, C, act_o, M, x, bias=v["b_xout"], out=x,
                                           stream=stream)
        act2 = b2q.norm_modulate_q8(x, 1e-6, v["scale_mlp"], v["shift_mlp"], stream=stream)
        act3 = b2q.mul_mat_prepared_gelu_q8(self.packed["fc1"], self.hidden, C, act2, M, bias=v["b1"],
                                            stream=stream)
        b2q.mul_mat_prepared_gate_residual(self.packed["fc2"], C, self.hidden, act3, M, x, bias=v["b2"],
                                           gate=v["gate_mlp"], out=x, stream=stream)
        return x
