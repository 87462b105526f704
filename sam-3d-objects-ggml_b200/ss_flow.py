"""The sparse-structure flow DiT on the device: the model forward of
cpp_ggml/src/ss_flow_graph.cpp:56-419 and one Euler / CFG sampling step of
cpp_ggml/src/session.cpp:1199-1245, composed from libb2q's entry points.

Forward (the two CFG branches of one object run batched, B = 2, where the
reference runs its graph twice; the unconditional branch feeds zero condition
tokens and both feed d = 0, session.cpp:1137-1139):

    mod   = E_t(t) + E_d(d)            E(s) = Lin(SiLU(Lin(cos(s f) | sin(s f))))     :134-158
    six_i = SiLU(mod) . W_adaLN_i + b_i  for every block i                              :179-185
    hs    = x_shape . W_in + b + pos_emb            (n_shape tokens, F32 weights, K=8)  :162-169
    hp    = the 4 pose tokens (6drotation, translation, scale, translation_scale),
            each from its own F32 input layer                                           :170-176
    per block, each group with its own weights and the block's shared modulation:
      self-attention: the shape group attends itself, the pose group attends the
        pose and shape keys                                                            :198-295
      cross-attention to the condition tokens                                          :297-354
      MLP (LN + modulate, fc1, GELU-tanh, fc2, gated residual)                          :356-385
    out   = LayerNorm -> out_layer per modality                                         :389-419

Step: v = vc + 7 (vc - vu) for every output while t*1000 lies in [0, 500], else
v = vc; then x += dt * v (session.cpp:1206-1242).

B200-first choices: the CFG branches share one pass (twice the tokens per
GEMM); the adaLN weights of all blocks are stacked into one [blocks*6C, C]
mul_mat (its input SiLU(mod) is the same for every block); the condition
tokens are quantized once per forward for all blocks and both groups; the
pose group runs on a second stream beside the shape group; the whole step is
captured into one CUDA graph (`capture`), both streams included.  The attention
cores are libb2q's (tensor-core fp16 form, or the F32 contract).  Torch pieces,
not the mul_mat path: the F32 input layers (K <= 8, not block-quantizable: torch
matmul), the timestep embedding's cos / sin and SiLU on 256 / 1024 values, and
the Euler update (torch elementwise).
"""
from __future__ import annotations

import math

import b2q

POSE = (("6drotation_normalized", 6), ("translation", 3), ("scale", 3), ("translation_scale", 1))
GROUPS = ("s", "p")  # shape group, pose group
CFG_STRENGTH, CFG_START, CFG_END = 7.0, 0.0, 500.0  # session.cpp:1048-1052
EPS = 1e-6


def linear_shapes(C: int, hidden: int) -> dict:
    """(out, in) of each per-group linear of a block."""
    return {"qkv": (3 * C, C), "out": (C, C), "xq": (C, C), "xkv": (2 * C, C), "xout": (C, C),
            "fc1": (hidden, C), "fc2": (C, hidden)}


def param_specs(C: int = 1024, n_blocks: int = 24, n_shape: int = 4096, in_ch: int = 8,
                mlp_ratio: int = 4) -> list:
    """Every parameter as (name, kind, shape, (mean, std)): kind "q" is a
    block-quantized linear weight [out, in] (GGUF rows), "f" an fp32 tensor."""
    hidden = C * mlp_ratio
    w, b = (0.0, 0.02), (0.0, 0.02)
    specs = []
    for e in ("t", "d"):
        specs += [(f"{e}.0", "q", (C, 256), w), (f"{e}.0.b", "f", (C,), b),
                  (f"{e}.2", "q", (C, C), w), (f"{e}.2.b", "f", (C,), b)]
    specs += [("in.shape", "f", (C, in_ch), (0.0, 0.3)), ("in.shape.b", "f", (C,), b),
              ("pe.shape", "f", (n_shape, C), (0.0, 0.5)),
              ("out.shape", "q", (in_ch, C), w), ("out.shape.b", "f", (in_ch,), b)]
    for m, ch in POSE:
        specs += [(f"in.{m}", "f", (C, ch), (0.0, 0.3)), (f"in.{m}.b", "f", (C,), b),
                  (f"pe.{m}", "f", (1, C), (0.0, 0.5)),
                  (f"out.{m}", "q", (ch, C), w), (f"out.{m}.b", "f", (ch,), b)]
    for i in range(n_blocks):
        specs += [(f"b{i}.adaln", "q", (6 * C, C), w), (f"b{i}.adaln.b", "f", (6 * C,), b)]
        for g in GROUPS:
            for name, shp in linear_shapes(C, hidden).items():
                specs += [(f"b{i}.{g}.{name}", "q", shp, w), (f"b{i}.{g}.{name}.b", "f", (shp[0],), b)]
            specs += [(f"b{i}.{g}.gq", "f", (C,), (1.0, 0.1)), (f"b{i}.{g}.gk", "f", (C,), (1.0, 0.1)),
                      (f"b{i}.{g}.n2w", "f", (C,), (1.0, 0.1)), (f"b{i}.{g}.n2b", "f", (C,), (0.0, 0.1))]
    return specs


def random_params(specs: list, dev, wtype: int = b2q.TYPE_Q8_0, seed: int = 0) -> dict:
    """Random-init parameters generated on the device: fp32 tensors from their
    (mean, std); quantized weights as valid GGUF rows whose codes and fp16
    scales have the magnitudes of N(0, std) quantized (benchmark weights)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for name, kind, shape, (mean, std) in specs:
        if kind == "f":
            out[name] = torch.randn(shape, generator=g, device=dev) * std + mean
            continue
        n, k = shape
        nb = k // 32
        amax = (torch.rand((n, nb), generator=g, device=dev) * 0.5 + 0.75) * (3.0 * std)  # block |max|
        if wtype == b2q.TYPE_Q8_0:
            codes = torch.randint(-127, 128, (n, nb, 32), generator=g, device=dev, dtype=torch.int8)
            d = amax / 127.0
            payload = codes.view(torch.uint8)
        elif wtype == b2q.TYPE_Q4_0:
            payload = torch.randint(0, 256, (n, nb, 16), generator=g, device=dev, dtype=torch.uint8)
            d = amax / 8.0
        else:
            raise ValueError("random_params: Q8_0 or Q4_0 weights")
        dbytes = d.to(torch.float16).contiguous().view(torch.uint8).view(n, nb, 2)
        out[name] = torch.cat([dbytes, payload], dim=2).reshape(n, -1).contiguous()
    return out


class SsFlow:
    """Packed weights of the whole SS-flow DiT and its forward / sampling step."""

    def __init__(self, dev, params: dict, C: int = 1024, heads: int = 16, n_blocks: int = 24,
                 n_shape: int = 4096, in_ch: int = 8, mlp_ratio: int = 4, wtype: int = b2q.TYPE_Q8_0,
                 attn: str = "f16"):
        """params: name -> tensor per param_specs (numpy or torch): "q" entries
        GGUF rows of wtype, uint8 [out, row bytes]; "f" entries fp32.
        attn: "f16" -- the production attention (q, k, v and o in fp16, the
        reference's flash-attention path with F16 K/V); "f32" -- the reference's
        F32 numeric-gate contract (gb_attention with strict K/V,
        cpp_ggml/src/graph_builder.cpp:139-175): fp32 heads, libb2q's fp32
        online-softmax core, fp32 output into the projection."""
        import numpy as np
        import torch
        if attn not in ("f16", "f32"):
            raise ValueError("attn: 'f16' or 'f32'")
        self.attn = attn
        self.dev, self.C, self.H, self.D = dev, C, heads, C // heads
        self.nb, self.T, self.in_ch, self.hidden, self.wtype = n_blocks, n_shape, in_ch, C * mlp_ratio, wtype

        def dev_t(a, dtype=None):
            t = torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a
            return t.to(device=dev, dtype=dtype).contiguous()

        self.W, self.V = {}, {}
        stacked = []
        for name, kind, shape, _ in param_specs(C, n_blocks, n_shape, in_ch, mlp_ratio):
            if kind == "f":
                self.V[name] = dev_t(params[name], torch.float32).reshape(shape)
            elif name.endswith(".adaln"):
                stacked.append(dev_t(params[name], torch.uint8))
            else:
                self.W[name] = b2q.weight_pack(wtype, dev_t(params[name], torch.uint8), shape[1])
        # adaLN of every block as one [blocks*6C, C] matrix: GGUF rows stack.
        self.W_adaln = b2q.weight_pack(wtype, torch.cat(stacked, 0), C)
        self.b_adaln = torch.cat([self.V[f"b{i}.adaln.b"] for i in range(n_blocks)])
        # timestep frequencies, as the reference fills its table on the host (fp32)
        half = 128
        f = np.exp(np.float32(-math.log(10000.0)) * np.arange(half, dtype=np.float32) / np.float32(half))
        self.freqs = torch.from_numpy(f.astype(np.float32)).to(dev)

    # ------------------------------------------------------------ pieces
    def _embed(self, e: str, s):
        import torch
        import torch.nn.functional as F
        C = self.C
        ang = s * self.freqs
        emb = torch.cat([torch.cos(ang), torch.sin(ang)]).reshape(1, 256)
        h = b2q.mul_mat_packed(self.W[f"{e}.0"], C, 256, emb, bias=self.V[f"{e}.0.b"])
        return b2q.mul_mat_packed(self.W[f"{e}.2"], C, C, F.silu(h), bias=self.V[f"{e}.2.b"])

    def _qkv(self, g: str, i: int, x, B: int, T: int, scale, shift):
        C, H, D, p = self.C, self.H, self.D, f"b{i}.{g}."
        act = b2q.norm_modulate_q8(x, EPS, scale, shift)
        qkv = b2q.mul_mat_prepared(self.W[p + "qkv"], 3 * C, C, act, B * T, bias=self.V[p + "qkv.b"])
        heads = b2q.qkv_heads_f32 if self.attn == "f32" else b2q.qkv_heads
        return heads(qkv, B, T, H, D, self.V[p + "gq"], self.V[p + "gk"], EPS)

    def _attend(self, q, k, v, k2=None, v2=None):
        """The attention core, its output as the to_out linear's Q8_0 prepared
        activations: fp16 heads -> libb2q's tensor-core attention with the
        quantize in its epilogue (production; the bytes of heads_act_prepare of
        its fp16 rows), or fp32 heads -> fp32 rows [B*T, C] -> act_prepare (F32
        contract).  k2 / v2: a second key source appended after k / v."""
        if self.attn == "f32":
            return b2q.act_prepare(b2q.attention_f32(q, k, v, k2, v2))
        return b2q.attention_f16_q8(q, k, v, k2, v2)

    def _attn_out(self, g: str, i: int, act, x, gate, name: str = "out"):
        p = f"b{i}.{g}.{name}"
        b2q.mul_mat_prepared_gate_residual(self.W[p], self.C, self.C, act, x.shape[0], x, bias=self.V[p + ".b"],
                                           gate=gate, out=x)

    def _cross(self, g: str, i: int, x, B: int, T: int, act_c, n_cond: int):
        C, H, D, p = self.C, self.H, self.D, f"b{i}.{g}."
        act = b2q.layer_norm_q8(x, EPS, self.V[p + "n2w"], self.V[p + "n2b"])
        if self.attn == "f16" and D == 64:
            # the projections' tile ends write the fp16 heads (the few-token q keeps
            # the two-step form: its GEMM runs on the CUDA cores)
            if B * T > b2q.GEMV_MAX_M:
                (q,) = b2q.mul_mat_prepared_heads(self.W[p + "xq"], C, C, act, B, T, H, D, bias=self.V[p + "xq.b"])
            else:
                xq = b2q.mul_mat_prepared(self.W[p + "xq"], C, C, act, B * T, bias=self.V[p + "xq.b"])
                (q,) = b2q.rows_to_heads(xq, B, T, H, D, 1)
            k, v = b2q.mul_mat_prepared_heads(self.W[p + "xkv"], 2 * C, C, act_c, B, n_cond, H, D,
                                              bias=self.V[p + "xkv.b"])
        else:
            xq = b2q.mul_mat_prepared(self.W[p + "xq"], C, C, act, B * T, bias=self.V[p + "xq.b"])
            xkv = b2q.mul_mat_prepared(self.W[p + "xkv"], 2 * C, C, act_c, B * n_cond, bias=self.V[p + "xkv.b"])
            heads = b2q.rows_to_heads_f32 if self.attn == "f32" else b2q.rows_to_heads
            (q,) = heads(xq, B, T, H, D, 1)
            k, v = heads(xkv, B, n_cond, H, D, 2)
        self._attn_out(g, i, self._attend(q, k, v), x, None, "xout")

    def _mlp(self, g: str, i: int, x, scale, shift, gate):
        C, p = self.C, f"b{i}.{g}."
        act = b2q.norm_modulate_q8(x, EPS, scale, shift)
        act = b2q.mul_mat_prepared_gelu_q8(self.W[p + "fc1"], self.hidden, C, act, x.shape[0], bias=self.V[p + "fc1.b"])
        b2q.mul_mat_prepared_gate_residual(self.W[p + "fc2"], C, self.hidden, act, x.shape[0], x,
                                           bias=self.V[p + "fc2.b"], gate=gate, out=x)

    # ------------------------------------------------------------ forward
    def forward(self, xs, xp: dict, t, d, cond, B: int):
        """Velocities of B branches.  xs: fp32 [B*n_shape, in_ch]; xp: pose
        modality -> fp32 [B, ch]; t, d: fp32 device [1] (t already x1000);
        cond: fp32 [B*n_cond, C].  Returns (v_shape [B*n_shape, in_ch],
        {modality: [B, ch]})."""
        import torch
        import torch.nn.functional as F
        C, T, nb = self.C, self.T, self.nb
        n_cond = cond.shape[0] // B
        main = torch.cuda.current_stream(self.dev)
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.dev)
        side = self._side
        mod = self._embed("t", t) + self._embed("d", d)
        six_all = b2q.mul_mat_packed(self.W_adaln, nb * 6 * C, C, F.silu(mod), bias=self.b_adaln)
        act_c = b2q.act_prepare(cond)  # one quantize of the condition tokens for every block and group
        # input projections (F32 weights, K <= 8)
        hs = (xs @ self.V["in.shape"].t() + self.V["in.shape.b"]).view(B, T, C)
        hs = (hs + self.V["pe.shape"]).view(B * T, C).contiguous()
        hp = torch.stack([xp[m] @ self.V[f"in.{m}"].t() + self.V[f"in.{m}.b"] + self.V[f"pe.{m}"][0]
                          for m, _ in POSE], 1).reshape(B * 4, C).contiguous()  # row b*4 + j
        # The 4-token pose group runs on a second stream: its kernels are small
        # and latency-bound, and only its self-attention needs the shape
        # group's keys and values (one event per block).  The shape group keeps
        # the main stream; both join before the output layers.
        forked = torch.cuda.Event()
        forked.record(main)
        side.wait_event(forked)
        for t_ in (six_all, act_c, hp):
            t_.record_stream(side)
        for i in range(nb):
            six = six_all[0, i * 6 * C:(i + 1) * 6 * C]
            shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (six[j * C:(j + 1) * C]
                                                                              for j in range(6))
            qs, ks, vs = self._qkv("s", i, hs, B, T, scale_msa, shift_msa)
            kv_ready = torch.cuda.Event()
            kv_ready.record(main)
            with torch.cuda.stream(side):
                qp, kp, vp = self._qkv("p", i, hp, B, 4, scale_msa, shift_msa)
                side.wait_event(kv_ready)
                ks.record_stream(side)
                vs.record_stream(side)
                o_p = self._attend(qp, kp, vp, ks, vs)
                self._attn_out("p", i, o_p, hp, gate_msa)
                self._cross("p", i, hp, B, 4, act_c, n_cond)
                self._mlp("p", i, hp, scale_mlp, shift_mlp, gate_mlp)
            o_s = self._attend(qs, ks, vs)
            self._attn_out("s", i, o_s, hs, gate_msa)
            self._cross("s", i, hs, B, T, act_c, n_cond)
            self._mlp("s", i, hs, scale_mlp, shift_mlp, gate_mlp)
        joined = torch.cuda.Event()
        joined.record(side)
        main.wait_event(joined)
        act = b2q.norm_modulate_q8(hs, EPS)
        v_shape = b2q.mul_mat_prepared(self.W["out.shape"], self.in_ch, C, act, B * T, bias=self.V["out.shape.b"])
        hpn = b2q.norm_modulate(hp, EPS)
        v_pose = {m: b2q.mul_mat_packed(self.W[f"out.{m}"], ch, C, hpn[j::4], bias=self.V[f"out.{m}.b"])
                  for j, (m, ch) in enumerate(POSE)}
        return v_shape, v_pose


class SsSampler:
    """One object's SS sampling state on the device and its Euler / CFG step,
    optionally captured into a CUDA graph.  The step's inputs (model time,
    dt) live in device scalars so a captured graph replays every step."""

    def __init__(self, flow: SsFlow, cond, n_cond: int, seed: int = 0):
        """cond: fp32 [n_cond, C] condition tokens of this object."""
        import torch
        dev, C = flow.dev, flow.C
        self.flow, self.n_cond = flow, n_cond
        g = torch.Generator(device=dev).manual_seed(seed)
        self.xs = torch.randn(flow.T, flow.in_ch, generator=g, device=dev)  # noise at t = 0
        self.xp = {m: torch.randn(1, ch, generator=g, device=dev) for m, ch in POSE}
        self.cond2 = torch.zeros(2 * n_cond, C, device=dev)  # [cond; zeros] for the CFG pair
        self.cond2[:n_cond].copy_(cond)
        self.t = torch.zeros(1, device=dev)
        self.d = torch.zeros(1, device=dev)
        self.dt = torch.zeros(1, device=dev)
        self.graphs = {}

    def _step(self, cfg: bool):
        B = 2 if cfg else 1
        f = self.flow
        xs = self.xs.repeat(B, 1)
        xp = {m: v.repeat(B, 1) for m, v in self.xp.items()}
        vs, vp = f.forward(xs, xp, self.t, self.d, self.cond2[:B * self.n_cond], B)

        def update(x, v, rows):
            vc = v[:rows]
            if cfg:
                vc = vc + CFG_STRENGTH * (vc - v[rows:])
            x.add_(self.dt * vc)

        update(self.xs, vs, f.T)
        for m, _ in POSE:
            update(self.xp[m], vp[m], 1)

    def step(self, t_model: float, dt: float):
        """One Euler step at model time t_model (= t * 1000)."""
        cfg = CFG_START <= t_model <= CFG_END
        self.t.fill_(t_model)
        self.dt.fill_(dt)
        g = self.graphs.get(cfg)
        if g is None:
            self._step(cfg)
        else:
            g.replay()

    def capture(self, cfg: bool = True):
        """Record one step into a CUDA graph.  One eager warm-up step runs first
        on a side stream with dt = 0, so the state does not move."""
        import torch
        dt = self.dt.clone()
        self.dt.zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step(cfg)
        torch.cuda.current_stream().wait_stream(s)
        self.dt.copy_(dt)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):  # other threads (e.g. a NCCL watchdog) may query events
            self._step(cfg)
        self.graphs[cfg] = g
        return g


def euler_schedule(steps: int = 25, rescale_t: float = 3.0) -> list:
    """(t, dt) per step: t_i = u / (1 + (r - 1)(1 - u)), u = i / steps, in
    double then rounded to fp32 (session.cpp:129-148)."""
    import numpy as np
    ts = []
    for i in range(steps + 1):
        u = i / steps
        ts.append(np.float32(u / (1.0 + (rescale_t - 1.0) * (1.0 - u)) if rescale_t != 0.0 else u))
    return [(float(ts[i]), float(np.float32(ts[i + 1] - ts[i]))) for i in range(steps)]
