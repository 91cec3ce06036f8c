"""GPU parity tests of matvec chains (tq_chain_create / tq_chain_run): one
launch running dependent single-row matvecs in order, with the RMSNorm
prologue and the SwiGLU / residual epilogues fused in.

Every op's output is checked against the CPU oracle applied to that op's own
GPU input (the AVX2 restatement of quant_simd.go / quant4_simd.go), within the
matvec bar of 1e-5 relative L2; norms and epilogues against a float64 / float32
restatement of _example/qwen/model.go:182-193, 276-278, 296-303. At the int4
MLP sizes two launches of a chain agree bit for bit and the single-call
kernel agrees to the matvec bar.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import _lib
from tensai_b200 import quant as Q

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


def make(bits, rows, cols, seed, stream):
    """A resident matrix quantized from seeded weights, plus the oracle's codes."""
    import torch
    w = O.synth((rows, cols), seed, stream, 0.02)
    wd = torch.from_numpy(w).cuda()
    h = Q.quantize_dev(wd, bits)
    torch.cuda.synchronize()
    q, s = Q.download(h, bits, rows, cols)
    qo, so = (O.quantize8 if bits == 8 else O.quantize4)(w)
    assert np.array_equal(q, qo) and np.array_equal(s.view(np.uint32), so.view(np.uint32))
    return h, q, s


def oracle_mv(bits, q, s, rows, cols, x):
    return (O.q8_matmul if bits == 8 else O.q4_matmul)(q, s, rows, cols, x)[0]


def rmsnorm(x, w, eps):
    """model.go:182-193: float64 sum of squares, out = float32(float64(x) * inv) * w."""
    x64 = x.astype(np.float64)
    inv = 1.0 / np.sqrt(np.dot(x64, x64) / x.size + eps)
    return (x64 * inv).astype(np.float32) * w


def swiglu(g):
    f = g.size // 2
    gd = g[:f].astype(np.float64)
    return (gd / (1.0 + np.exp(-gd))).astype(np.float32) * g[f:]


def dev(n):
    import torch
    # 16-byte aligned (torch's allocator aligns to 512 B)
    return torch.zeros(n, device="cuda", dtype=torch.float32)


# (bits, [(rows, cols), ...]): each op's rows equal the previous op's cols.
PLAIN = [
    (4, [(4096, 11008), (11008, 4096), (4096, 11008), (11008, 4096)]),
    (4, [(200, 130), (130, 66), (66, 1030), (1030, 2), (2, 256)]),
    (4, [(33, 10), (10, 4096), (4096, 98)]),
    (8, [(768, 2304), (2304, 768), (768, 3072), (3072, 768)]),
    (8, [(300, 1031), (1031, 77), (77, 5), (5, 129)]),
]


@pytest.mark.parametrize("bits,shapes", PLAIN, ids=[f"int{b}-{len(s)}ops-{s[0][0]}x{s[0][1]}" for b, s in PLAIN])
def test_chain_matches_oracle_per_op(bits, shapes):
    import torch
    mats = [make(bits, r, c, 11, 40 + i) for i, (r, c) in enumerate(shapes)]
    x0 = O.synth((shapes[0][0],), 11, 1, 1.0)
    bufs = [torch.from_numpy(x0).cuda()] + [dev(c) for _, c in shapes]
    ops = [{"handle": mats[i][0], "x": bufs[i], "out": bufs[i + 1]} for i in range(len(shapes))]
    with Q.Chain(ops) as ch:
        for rep in range(3):  # counters re-arm between launches
            for b in bufs[1:]:
                b.fill_(float("nan"))
            ch.run()
            torch.cuda.synchronize()
            for i, (r, c) in enumerate(shapes):
                xin = bufs[i].cpu().numpy()
                got = bufs[i + 1].cpu().numpy()
                want = oracle_mv(bits, mats[i][1], mats[i][2], r, c, xin)
                assert np.isfinite(got).all(), (rep, i)
                assert rel_l2(got, want) <= REL_L2, (rep, i, rel_l2(got, want))
    for h, _, _ in mats:
        Q.free(h)


def test_chain_int4_reproducible_and_close_to_single_calls():
    """The MLP pair at M=1: the int4 chain (column-owner CTAs) adds each
    column's groups in its own fixed order, so two launches agree bit for bit
    and the single-call kernel (a different split) agrees to the matvec bar."""
    import torch
    shapes = [(4096, 11008), (11008, 4096)]
    mats = [make(4, r, c, 12, 60 + i) for i, (r, c) in enumerate(shapes)]
    x0 = torch.from_numpy(O.synth((4096,), 12, 1, 1.0)).cuda()
    h1, o1 = dev(11008), dev(4096)
    with Q.Chain([{"handle": mats[0][0], "x": x0, "out": h1}, {"handle": mats[1][0], "x": h1, "out": o1}]) as ch:
        ch.run()
        torch.cuda.synchronize()
        first = (h1.clone(), o1.clone())
        h1.fill_(float("nan"))
        o1.fill_(float("nan"))
        ch.run()
        torch.cuda.synchronize()
        assert torch.equal(h1, first[0]) and torch.equal(o1, first[1])
        h2, o2 = dev(11008), dev(4096)
        Q.matmul_dev(mats[0][0], x0.view(1, -1), h2.view(1, -1))
        Q.matmul_dev(mats[1][0], h1.view(1, -1), o2.view(1, -1))
        torch.cuda.synchronize()
        assert rel_l2(h1.cpu().numpy(), h2.cpu().numpy()) <= REL_L2
        assert rel_l2(o1.cpu().numpy(), o2.cpu().numpy()) <= REL_L2
    for h, _, _ in mats:
        Q.free(h)


def test_chain_ops_without_a_direct_dependency_keep_call_order():
    """Op 1 reads an external input and overwrites op 0's input; op 2 reads
    op 0's output (not op 1's) and op 3 a prefix of op 2's output: each must
    see what consecutive calls would see."""
    import torch
    shapes = [(512, 768), (256, 512), (768, 640), (320, 192)]
    mats = [make(4, r, c, 15, 90 + i) for i, (r, c) in enumerate(shapes)]
    a0 = O.synth((512,), 15, 1, 1.0)
    c0 = O.synth((256,), 15, 2, 1.0)
    a, cbuf = torch.from_numpy(a0).cuda(), torch.from_numpy(c0).cuda()
    b, d, e = dev(768), dev(640), dev(192)
    ops = [
        {"handle": mats[0][0], "x": a, "out": b},     # b = a W0
        {"handle": mats[1][0], "x": cbuf, "out": a},  # a = c W1 (after op 0 read a)
        {"handle": mats[2][0], "x": b, "out": d},     # d = b W2 (b from op 0)
        {"handle": mats[3][0], "x": d, "out": e},     # e = d[:320] W3
    ]
    with Q.Chain(ops) as ch:
        for rep in range(3):
            a.copy_(torch.from_numpy(a0))
            ch.run()
            torch.cuda.synchronize()
            want_b = oracle_mv(4, mats[0][1], mats[0][2], 512, 768, a0)
            assert rel_l2(b.cpu().numpy(), want_b) <= REL_L2, rep
            want_a = oracle_mv(4, mats[1][1], mats[1][2], 256, 512, c0)
            assert rel_l2(a.cpu().numpy(), want_a) <= REL_L2, rep
            want_d = oracle_mv(4, mats[2][1], mats[2][2], 768, 640, b.cpu().numpy())
            assert rel_l2(d.cpu().numpy(), want_d) <= REL_L2, rep
            want_e = oracle_mv(4, mats[3][1], mats[3][2], 320, 192, d.cpu().numpy()[:320])
            assert rel_l2(e.cpu().numpy(), want_e) <= REL_L2, rep
    for h, _, _ in mats:
        Q.free(h)


def qwen_like_chain(d, f, n_out, seed, in_place):
    """o_proj (+residual), norm + gate|up (SwiGLU), down (+residual),
    norm + next projection: the ops of one decode layer."""
    import torch
    mo = make(4, d, d, seed, 1)
    mgu = make(4, d, 2 * f, seed, 2)
    md = make(4, f, d, seed, 3)
    mq = make(4, d, n_out, seed, 4)
    att = torch.from_numpy(O.synth((d,), seed, 10, 1.0)).cuda()
    x0 = O.synth((d,), seed, 11, 1.0)
    w1 = O.synth((d,), seed, 12, 0.3) + np.float32(1.0)
    w2 = O.synth((d,), seed, 13, 0.3) + np.float32(1.0)
    w1d, w2d = torch.from_numpy(w1).cuda(), torch.from_numpy(w2).cuda()
    xres = torch.from_numpy(x0).cuda()
    x1 = xres if in_place else dev(d)
    h = dev(f)
    x2 = xres if in_place else dev(d)
    out = dev(n_out)
    eps = 1e-6
    ops = [
        {"handle": mo[0], "x": att, "out": x1, "epilogue": "resid", "resid": xres},
        {"handle": mgu[0], "x": x1, "out": h, "epilogue": "swiglu", "norm_w": w1d, "norm_from": 0, "eps": eps},
        {"handle": md[0], "x": h, "out": x2, "epilogue": "resid", "resid": x1},
        {"handle": mq[0], "x": x2, "out": out, "norm_w": w2d, "norm_from": 2, "eps": eps},
    ]
    mats = (mo, mgu, md, mq)
    return ops, mats, dict(att=att, x0=x0, w1=w1, w2=w2, x1=x1, h=h, x2=x2, out=out, xres=xres, eps=eps)


@pytest.mark.parametrize("d,f,n_out", [(3584, 18944, 4608), (256, 512, 130), (192, 66, 2)])
def test_chain_norm_swiglu_residual(d, f, n_out):
    import torch
    ops, mats, b = qwen_like_chain(d, f, n_out, 21, in_place=False)
    mo, mgu, md, mq = mats
    with Q.Chain(ops) as ch:
        ch.run()
        torch.cuda.synchronize()
    att = b["att"].cpu().numpy()
    x1 = b["x1"].cpu().numpy()
    h = b["h"].cpu().numpy()
    x2 = b["x2"].cpu().numpy()
    out = b["out"].cpu().numpy()
    # o_proj + residual (float32 add)
    want_x1 = b["x0"] + oracle_mv(4, mo[1], mo[2], d, d, att)
    assert rel_l2(x1, want_x1) <= REL_L2
    # norm + gate|up + SwiGLU, from the GPU's x1
    want_h = swiglu(oracle_mv(4, mgu[1], mgu[2], d, 2 * f, rmsnorm(x1, b["w1"], b["eps"])))
    assert rel_l2(h, want_h) <= REL_L2
    # down + residual
    want_x2 = x1 + oracle_mv(4, md[1], md[2], f, d, h)
    assert rel_l2(x2, want_x2) <= REL_L2
    # norm + next projection
    want = oracle_mv(4, mq[1], mq[2], d, n_out, rmsnorm(x2, b["w2"], b["eps"]))
    assert rel_l2(out, want) <= REL_L2
    for m in mats:
        Q.free(m[0])


def test_chain_in_place_residual_equals_separate_buffers():
    """resid == out (x += o, as the decode step updates its residual stream)
    gives the same bits as separate buffers."""
    import torch
    outs = []
    for in_place in (False, True):
        ops, mats, b = qwen_like_chain(512, 1024, 300, 22, in_place)
        with Q.Chain(ops) as ch:
            ch.run()
            torch.cuda.synchronize()
        outs.append((b["x2"].clone(), b["out"].clone()))
        for m in mats:
            Q.free(m[0])
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])


def test_chain_in_cuda_graph_replays():
    import torch
    shapes = [(1024, 2048), (2048, 1024), (1024, 512)]
    mats = [make(4, r, c, 13, 80 + i) for i, (r, c) in enumerate(shapes)]
    bufs = [torch.from_numpy(O.synth((1024,), 13, 1, 1.0)).cuda()] + [dev(c) for _, c in shapes]
    ops = [{"handle": mats[i][0], "x": bufs[i], "out": bufs[i + 1]} for i in range(3)]
    st = torch.cuda.Stream()
    with Q.Chain(ops) as ch:
        with torch.cuda.stream(st):
            ch.run(st)  # the stream's scratch is made outside the capture
        torch.cuda.synchronize()
        ref = bufs[-1].clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            ch.run(st)
        for _ in range(5):
            bufs[-1].fill_(0.0)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(bufs[-1], ref)
        del g
    for h, _, _ in mats:
        Q.free(h)


def test_chain_rejects_bad_ops():
    import torch
    L = _lib.load()
    h4, _, _ = make(4, 128, 256, 14, 1)
    h8, _, _ = make(8, 256, 64, 14, 2)
    x = dev(256)
    y = dev(256)

    def code(ops):
        try:
            Q.Chain(ops).free()
            return 0, ""
        except _lib.TensaiError as e:
            return e.code, str(e)

    # mixed bit widths
    r = code([{"handle": h4, "x": x, "out": y}, {"handle": h8, "x": y, "out": x}])
    assert r[0] == _lib.TQ_ERR_ARG and "op 1" in r[1]
    # an input that is not 16-byte aligned
    r = code([{"handle": h4, "x": x.data_ptr() + 4, "out": y}])
    assert r[0] == _lib.TQ_ERR_ARG and "aligned" in r[1]
    # a norm whose source is not an earlier residual op
    r = code([{"handle": h4, "x": x, "out": y, "norm_w": x, "norm_from": 0}])
    assert r[0] == _lib.TQ_ERR_ARG and "normalised" in r[1]
    # SwiGLU on int8
    r = code([{"handle": h8, "x": x, "out": y, "epilogue": "swiglu"}])
    assert r[0] == _lib.TQ_ERR_ARG
    # an input overlapping an earlier op's output without being exactly it
    z = dev(1024)
    r = code([{"handle": h4, "x": x, "out": z}, {"handle": h4, "x": z[4:], "out": y}])
    assert r[0] == _lib.TQ_ERR_ARG and "op 1" in r[1] and "overlaps" in r[1]
    # an int4 output over its own (external) input
    r = code([{"handle": h4, "x": z, "out": z}])
    assert r[0] == _lib.TQ_ERR_ARG and "overlap" in r[1]
    # an int4 op wider than 256 columns per SM
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    hw, _, _ = make(4, 64, 512 * sms + 64, 14, 3)
    big = dev(512 * sms + 64)
    r = code([{"handle": hw, "x": x, "out": big}])
    assert r[0] == _lib.TQ_ERR_ARG and "too many columns" in r[1]
    Q.free(hw)
    # a freed handle
    Q.free(h8)
    r = code([{"handle": h8, "x": x, "out": y}])
    assert r[0] == _lib.TQ_ERR_HANDLE
    # run / free of an unknown chain
    assert L.tq_chain_run(987654321, None) == _lib.TQ_ERR_HANDLE
    assert L.tq_chain_free(987654321) == _lib.TQ_OK
    Q.free(h4)
    torch.cuda.synchronize()
