"""The whole SS-flow DiT forward and its Euler / CFG step on the device
(ss_flow.py) against a CPU composition of the same graph
(cpp_ggml/src/ss_flow_graph.cpp:56-419, session.cpp:1199-1245) in which every
quantized linear is the oracle's mul_mat, on a small seeded model."""
import numpy as np
import pytest

import b2q
import oracle as O
import ss_flow

CFG = dict(C=256, heads=4, n_blocks=2, n_shape=64, in_ch=8, mlp_ratio=4)
N_COND = 40
TOL = 3e-3  # fp16 attention cores (both sides round q, k, v, P and o to fp16)
# The pose outputs are 2 values each after a Q8_0 linear: one code flip moves
# them by ~0.4%.  The CPU graph itself moves translation_scale by 3.7e-3 between
# fp16 and fp32 attention cores (q, k, v, o rounding only), so their bar sits
# above that sensitivity.
POSE_TOL = 1e-2


def make_params(wtype, seed=0, cfg=None):
    cfg = CFG if cfg is None else cfg
    rng = np.random.default_rng(seed)
    p = {}
    specs = ss_flow.param_specs(cfg["C"], cfg["n_blocks"], cfg["n_shape"], cfg["in_ch"], cfg["mlp_ratio"])
    for name, kind, shape, (mean, std) in specs:
        v = (rng.standard_normal(shape) * std + mean).astype(np.float32)
        p[name] = O.quantize(v, wtype) if kind == "q" else v
    return p


def cpu_forward(p, wtype, xs, xp, t, d, cond, B, cfg=None, n_cond=None, attn="f16"):
    """The reference graph on the CPU: oracle mul_mat (x86 activation
    quantizer) for every quantized linear, fp32 numpy elementwise, and an fp64
    softmax attention on q / k / v / o rounded to fp16 (attn "f16", the
    production flash path) or kept in fp32 (attn "f32", the reference's F32
    numeric-gate contract, cpp_ggml/src/graph_builder.cpp:139-175)."""
    cfg = CFG if cfg is None else cfg
    n_cond = N_COND if n_cond is None else n_cond
    C, H, T, nb = cfg["C"], cfg["heads"], cfg["n_shape"], cfg["n_blocks"]
    D = C // H
    rnd = (lambda a: a.astype(np.float16).astype(np.float64)) if attn == "f16" else (lambda a: a.astype(np.float64))  # noqa: E731
    f32 = np.float32
    lin = lambda name, x: O.mul_mat(wtype, p[name], np.ascontiguousarray(x, f32), O.ACT_X86) + p[name + ".b"]  # noqa: E731
    silu = lambda x: (x / (f32(1) + np.exp(-x))).astype(f32)  # noqa: E731
    ln = lambda x: O.norm_modulate(x, 1e-6)  # noqa: E731
    modulate = lambda x, s, sh: O.norm_modulate(x, 1e-6, s, sh)  # noqa: E731

    half = 128
    freqs = np.exp(f32(-np.log(10000.0)) * np.arange(half, dtype=f32) / f32(half)).astype(f32)

    def embed(e, s):
        ang = (f32(s) * freqs).astype(f32)
        emb = np.concatenate([np.cos(ang), np.sin(ang)]).astype(f32)[None]
        return lin(f"{e}.2", silu(lin(f"{e}.0", emb)))

    mod = embed("t", t) + embed("d", d)
    sm = silu(mod)
    hs = ((xs @ p["in.shape"].T).astype(f32) + p["in.shape.b"]).reshape(B, T, C) + p["pe.shape"]
    hs = hs.reshape(B * T, C).astype(f32)
    hp = np.stack([(xp[m] @ p[f"in.{m}"].T).astype(f32) + p[f"in.{m}.b"] + p[f"pe.{m}"][0]
                   for m, _ in ss_flow.POSE], 1).reshape(B * 4, C).astype(f32)

    def heads(x, n, g=None):
        x = x.reshape(B, n, H, D)
        if g is not None:
            ms = ((x.astype(np.float64) ** 2).sum(-1, keepdims=True) / D).astype(f32)
            x = (x * (f32(1) / np.sqrt(ms + f32(1e-6)))).astype(f32) * g.reshape(H, D)
        return rnd(x).transpose(0, 2, 1, 3)

    def attend(q, k, v):
        s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(D)
        s = np.exp(s - s.max(-1, keepdims=True))
        if attn == "f16":  # the flash kernel's P operand is fp16; its row sum adds those fp16 values
            s = rnd(s)
        o = (s @ v) / s.sum(-1, keepdims=True)
        return rnd(o).astype(f32).transpose(0, 2, 1, 3).reshape(-1, C)

    for i in range(nb):
        six = (O.mul_mat(wtype, p[f"b{i}.adaln"], sm, O.ACT_X86) + p[f"b{i}.adaln.b"])[0]
        sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = (six[j * C:(j + 1) * C] for j in range(6))
        qkv = {}
        for g, x, n in (("s", hs, T), ("p", hp, 4)):
            y = lin(f"b{i}.{g}.qkv", modulate(x, sc_msa, sh_msa))
            qkv[g] = (heads(y[:, :C], n, p[f"b{i}.{g}.gq"]), heads(y[:, C:2 * C], n, p[f"b{i}.{g}.gk"]),
                      heads(y[:, 2 * C:], n))
        qs, ks, vs = qkv["s"]
        qp, kp, vp = qkv["p"]
        o_s = attend(qs, ks, vs)
        o_p = attend(qp, np.concatenate([kp, ks], 2), np.concatenate([vp, vs], 2))
        hs = hs + lin(f"b{i}.s.out", o_s) * g_msa
        hp = hp + lin(f"b{i}.p.out", o_p) * g_msa
        out = []
        for g, x, n in (("s", hs, T), ("p", hp, 4)):
            h = ln(x) * p[f"b{i}.{g}.n2w"] + p[f"b{i}.{g}.n2b"]
            q = heads(lin(f"b{i}.{g}.xq", h), n)
            kv = lin(f"b{i}.{g}.xkv", cond)
            o = attend(q, heads(kv[:, :C], n_cond), heads(kv[:, C:], n_cond))
            x = x + lin(f"b{i}.{g}.xout", o)
            h = O.gelu(lin(f"b{i}.{g}.fc1", modulate(x, sc_mlp, sh_mlp)))
            out.append(x + lin(f"b{i}.{g}.fc2", h) * g_mlp)
        hs, hp = out
    v_shape = lin("out.shape", ln(hs))
    hpn = ln(hp)
    v_pose = {m: lin(f"out.{m}", hpn[j::4]) for j, (m, _) in enumerate(ss_flow.POSE)}
    return v_shape, v_pose


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def inputs(B, seed=3, cfg=None, n_cond=None):
    cfg = CFG if cfg is None else cfg
    n_cond = N_COND if n_cond is None else n_cond
    rng = np.random.default_rng(seed)
    xs = np.repeat(rng.standard_normal((1, cfg["n_shape"], cfg["in_ch"])).astype(np.float32), B, 0)
    xs = xs.reshape(B * cfg["n_shape"], cfg["in_ch"])
    xp = {m: np.repeat(rng.standard_normal((1, ch)).astype(np.float32), B, 0) for m, ch in ss_flow.POSE}
    cond = rng.standard_normal((n_cond, cfg["C"])).astype(np.float32)
    cond2 = np.concatenate([cond, np.zeros_like(cond)])[:B * n_cond]
    return xs, xp, cond, cond2


@pytest.mark.gpu
@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
def test_flow_forward_matches_cpu_graph(b2q_mod, dev, wtype):
    import torch
    p = make_params(wtype)
    flow = ss_flow.SsFlow(dev, p, wtype=wtype, **CFG)
    B, t_model, d = 2, 412.5, 0.0
    xs, xp, _, cond2 = inputs(B)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    vs, vp = flow.forward(T(xs), {m: T(v) for m, v in xp.items()}, torch.tensor([t_model], device=dev),
                          torch.tensor([d], device=dev), T(cond2), B)
    torch.cuda.synchronize()
    rs, rp = cpu_forward(p, wtype, xs, xp, t_model, d, cond2, B)
    assert rel(vs.cpu().numpy(), rs) <= TOL
    for m, _ in ss_flow.POSE:
        assert rel(vp[m].cpu().numpy(), rp[m]) <= POSE_TOL, m
    assert b2q.device_status() == 0


@pytest.mark.gpu
def test_sampler_step_cfg_and_graph_replay(b2q_mod, dev):
    """One Euler step with CFG: the device update equals x + dt * (vc + 7 (vc -
    vu)) from the device's own velocities, and the CUDA-graph replay of the
    step is bit-identical to the eager step."""
    import torch
    wtype = O.TYPE_Q8_0
    p = make_params(wtype, seed=1)
    flow = ss_flow.SsFlow(dev, p, wtype=wtype, **CFG)
    _, _, cond, _ = inputs(2, seed=5)
    eager = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=9)
    graph = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=9)
    graph.capture(cfg=True)
    x0 = eager.xs.clone()
    xp0 = {m: v.clone() for m, v in eager.xp.items()}
    sched = ss_flow.euler_schedule()
    t, dt = sched[0]
    assert t * 1000.0 <= ss_flow.CFG_END
    # the step's velocities, computed directly
    vs, vp = flow.forward(x0.repeat(2, 1), {m: v.repeat(2, 1) for m, v in xp0.items()},
                          torch.tensor([t * 1000.0], device=dev), torch.zeros(1, device=dev), eager.cond2, 2)
    eager.step(t * 1000.0, dt)
    graph.step(t * 1000.0, dt)
    torch.cuda.synchronize()
    T_ = CFG["n_shape"]
    vc, vu = vs[:T_], vs[T_:]
    want = x0 + torch.tensor([dt], device=dev) * (vc + ss_flow.CFG_STRENGTH * (vc - vu))
    assert torch.equal(eager.xs, want)
    assert torch.equal(graph.xs, eager.xs)
    for m in eager.xp:
        assert torch.equal(graph.xp[m], eager.xp[m])
        vcm, vum = vp[m][:1], vp[m][1:]
        assert torch.equal(eager.xp[m], xp0[m] + torch.tensor([dt], device=dev) * (vcm + 7.0 * (vcm - vum)))
    assert not torch.equal(eager.xs, x0)
    assert b2q.device_status() == 0


def test_euler_schedule_matches_reference_formula():
    s = ss_flow.euler_schedule(25, 3.0)
    assert len(s) == 25 and s[0][0] == 0.0
    ts = [a for a, _ in s] + [s[-1][0] + s[-1][1]]
    assert all(b > a for a, b in zip(ts, ts[1:]))
    u = 0.52
    assert abs(np.float32(u / (1 + 2 * (1 - u))) - ss_flow.euler_schedule(50, 3.0)[26][0]) < 1e-7
    assert abs(sum(dt for _, dt in s) - 1.0) < 1e-5


@pytest.mark.gpu
def test_sampler_step_without_cfg(b2q_mod, dev):
    """A step past the CFG window (model time > 500) runs the conditional
    branch alone (B = 1) and integrates x + dt * vc; its captured graph
    replays bit-identically."""
    import torch
    wtype = O.TYPE_Q8_0
    p = make_params(wtype, seed=2)
    flow = ss_flow.SsFlow(dev, p, wtype=wtype, **CFG)
    _, _, cond, _ = inputs(1, seed=6)
    eager = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=4)
    graph = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=4)
    graph.capture(cfg=False)
    t, dt = ss_flow.euler_schedule()[20]
    assert t * 1000.0 > ss_flow.CFG_END
    x0 = eager.xs.clone()
    vs, vp = flow.forward(x0, {m: v.clone() for m, v in eager.xp.items()}, torch.tensor([t * 1000.0], device=dev),
                          torch.zeros(1, device=dev), eager.cond2[:N_COND], 1)
    eager.step(t * 1000.0, dt)
    graph.step(t * 1000.0, dt)
    torch.cuda.synchronize()
    assert torch.equal(eager.xs, x0 + torch.tensor([dt], device=dev) * vs)
    assert torch.equal(graph.xs, eager.xs)
    for m in eager.xp:
        assert torch.equal(graph.xp[m], eager.xp[m])
    assert b2q.device_status() == 0


@pytest.mark.gpu
def test_full_sampling_loop_graph_equals_eager(b2q_mod, dev):
    """The reference's whole SS sampling loop (25 rescaled Euler steps, CFG on
    the first half): replaying the two captured graphs gives bit for bit the
    eager loop's final state, and the state stays finite."""
    import torch
    wtype = O.TYPE_Q8_0
    p = make_params(wtype, seed=3)
    flow = ss_flow.SsFlow(dev, p, wtype=wtype, **CFG)
    _, _, cond, _ = inputs(1, seed=8)
    eager = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=11)
    graph = ss_flow.SsSampler(flow, torch.from_numpy(cond).to(dev), N_COND, seed=11)
    graph.capture(cfg=True)
    graph.capture(cfg=False)
    sched = ss_flow.euler_schedule()
    assert any(t * 1000.0 <= ss_flow.CFG_END for t, _ in sched) and any(t * 1000.0 > ss_flow.CFG_END for t, _ in sched)
    for t, dt in sched:
        eager.step(t * 1000.0, dt)
        graph.step(t * 1000.0, dt)
    torch.cuda.synchronize()
    assert torch.isfinite(eager.xs).all()
    assert torch.equal(graph.xs, eager.xs)
    for m in eager.xp:
        assert torch.equal(graph.xp[m], eager.xp[m])
    assert b2q.device_status() == 0
