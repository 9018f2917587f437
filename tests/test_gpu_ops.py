"""GPU parity of each kernel against the CPU oracle, through the C ABI.

Tolerances: bit-exact for the int8 format (quantise, dequantise, gather); f32 paths 1e-4 max relative error
(north_star's fp32-accumulation bound) or tighter; bf16 paths 2e-2 (north_star's bf16 bound)."""
import math

import numpy as np
import pytest
import torch

from conftest import rel_max
from oracle import mixer, q8 as oq8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda):
    from duo import ops as o
    return o


def _seed(s):
    return torch.Generator(device="cpu").manual_seed(s)


# ---------------------------------------------------------------------------------------------------------------
# int8 format (engine/kernels.js:16-47, 205-221): bit-exact


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,k,group", [(37, 256, 128), (5, 1024, 1024), (300, 384, 128), (1, 128, 128)])
def test_q8_quantize_bit_exact(ops, dtype, n, k, group):
    w = torch.randn(n, k, generator=_seed(n * 7 + k)) * 0.05
    w[0, :min(k, 128)] = 0.0                            # an all-zero group -> scale 1
    if k >= 256:
        w[-1, 128:256] = torch.arange(128) * 0.5 - 32.0  # exact halves under scale 0.5/127*... edge values
    w = w.to(dtype)
    q, s = ops.q8_quantize(w.cuda(), group)
    rq, rs = oq8.quantize(w.float().numpy(), group)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_q8_dequant_and_gather_exact(ops):
    w = torch.randn(500, 256, generator=_seed(3)) * 0.02
    q, s = ops.q8_quantize(w.cuda(), 128)
    d = ops.q8_dequantize(q, s, torch.float32)
    ref = oq8.dequantize(q.cpu().numpy(), s.cpu().numpy(), 128)
    assert np.array_equal(d.cpu().numpy(), ref)
    db = ops.q8_dequantize(q, s, torch.bfloat16)
    assert torch.equal(db.cpu(), torch.from_numpy(ref).to(torch.bfloat16))
    ids = torch.tensor([0, 499, 17, 17, 250], dtype=torch.int32)
    g = ops.q8_gather(ids.cuda(), q, s)
    assert np.array_equal(g.cpu().numpy(), oq8.gather(ids.numpy(), q.cpu().numpy(), s.cpu().numpy(), 128))


# ---------------------------------------------------------------------------------------------------------------
# decode GEMV (engine/kernels.js:55-94)


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("k,group", [(1024, 128), (3584, 128), (2048, 2048)])
def test_q8_gemv(ops, m, k, group):
    n = 1000
    w = torch.randn(n, k, generator=_seed(k + m)) * 0.02
    x = torch.randn(m, k, generator=_seed(k - m))
    q, s = ops.q8_quantize(w.cuda(), group)
    ref = oq8.matvec(x.numpy(), q.cpu().numpy(), s.cpu().numpy(), group)
    y = ops.q8_gemv(x.cuda(), q, s)
    assert rel_max(y, ref) < 1e-5
    # accumulate into an existing f32 output (the residual add)
    y0 = torch.randn(m, n, generator=_seed(5))
    y2 = ops.q8_gemv(x.cuda(), q, s, y=y0.clone().cuda(), accumulate=True)
    assert rel_max(y2, ref + y0.numpy()) < 1e-5
    # bf16 activations in and out
    yb = ops.q8_gemv(x.to(torch.bfloat16).cuda(), q, s, out_dtype=torch.bfloat16)
    refb = oq8.matvec(x.to(torch.bfloat16).float().numpy(), q.cpu().numpy(), s.cpu().numpy(), group)
    assert rel_max(yb.float(), refb) < 1e-2


@pytest.mark.parametrize("m", [1, 3])
@pytest.mark.parametrize("n,k,group", [(70000, 1024, 128), (33000, 2048, 2048)])
def test_q8_gemv_streaming(ops, m, n, k, group):
    """Matrices of the LM head's size class (grid-stride row groups, ragged last group)."""
    w = torch.randn(n, k, generator=_seed(n + m)) * 0.02
    x = torch.randn(m, k, generator=_seed(k + 7 * m))
    q, s = ops.q8_quantize(w.cuda(), group)
    ref = oq8.matvec(x.numpy(), q.cpu().numpy(), s.cpu().numpy(), group)
    assert rel_max(ops.q8_gemv(x.cuda(), q, s), ref) < 1e-5
    y0 = torch.randn(m, n, generator=_seed(6))
    y2 = ops.q8_gemv(x.cuda(), q, s, y=y0.clone().cuda(), accumulate=True)
    assert rel_max(y2, ref + y0.numpy()) < 1e-5
    assert ops.fault_status() == 0


def test_q8_gemv_streaming_alternating_sizes(ops):
    """One streaming kernel launched with a large, a small, then the large shared-memory ring again (k = 1024 and
    k = 256 give different ring sizes): the kernel's shared-memory limit must never be left below a size in use."""
    outs = []
    for n, k in [(4096, 1024), (2048, 256), (4096, 1024), (2048, 256)]:
        w = torch.randn(n, k, generator=_seed(n + k)) * 0.02
        x = torch.randn(1, k, generator=_seed(k))
        q, s = ops.q8_quantize(w.cuda(), 128)
        ref = oq8.matvec(x.numpy(), q.cpu().numpy(), s.cpu().numpy(), 128)
        outs.append(rel_max(ops.q8_gemv(x.cuda(), q, s), ref))
    assert max(outs) < 1e-5
    assert ops.fault_status() == 0


# ---------------------------------------------------------------------------------------------------------------
# tcgen05 GEMM vs a torch fp32 matmul of the same bf16 operands


# small grids run the per-tile kernel (K split for the residual add); (4173, 1064, 1024) and (8269, 2088, 512) run the
# persistent kernel with ragged edge tiles and one to four tiles per CTA
# m <= 256 runs the decode kernel: (256, 8224, 1024) and (77, 5120, 1024) without a K split (TMA-store epilogue, a
# ragged last weight block, a ragged row group), (100, 1024, 3584) and (256, 1024, 2048) with K split over a cluster
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 300, 1024), (1024, 1024, 3584), (40, 7168, 1024),
                                   (3000, 512, 2048), (4173, 1064, 1024), (8269, 2088, 512), (256, 8224, 1024),
                                   (77, 5120, 1024), (100, 1024, 3584), (256, 1024, 2048)])
def test_gemm_bf16(ops, m, n, k):
    a = (torch.randn(m, k, generator=_seed(m)) ).to(torch.bfloat16)
    b = (torch.randn(n, k, generator=_seed(n)) * 0.05).to(torch.bfloat16)
    ref = a.float() @ b.float().T
    c = ops.gemm_bf16(a.cuda(), b.cuda(), out_dtype=torch.float32)
    assert rel_max(c, ref) < 1e-5 * max(1.0, k / 1024)  # f32 summation order over k terms
    cb = ops.gemm_bf16(a.cuda(), b.cuda(), out_dtype=torch.bfloat16)
    assert rel_max(cb.float(), ref) < 8e-3
    cs = torch.rand(n, generator=_seed(1)) + 0.5
    x0 = torch.randn(m, n, generator=_seed(2))
    acc = ops.gemm_bf16(a.cuda(), b.cuda(), col_scale=cs.cuda(), out=x0.clone().cuda(), accumulate=True)
    assert rel_max(acc, x0 + ref * cs) < 1e-5 * max(1.0, k / 1024)
    assert ops.fault_status() == 0


@pytest.mark.parametrize("m,inter,k,dt", [(37, 128, 256, torch.bfloat16), (100, 3584, 1024, torch.bfloat16),
                                          (256, 3584, 1024, torch.bfloat16), (250, 3584, 1024, torch.float16),
                                          (1000, 3584, 1024, torch.bfloat16), (1000, 3584, 1024, torch.float16)])
def test_gemm_swiglu(ops, m, inter, k, dt):
    """Fused gate|up GEMM + SwiGLU + neuron pushes (kernels_qwen35.js:250-280) against the oracle on the same 16-bit
    operands; the 16-bit output rounding bounds the error (m = 1000 runs the persistent kernel, m = 250 / 256 the
    decode kernel's TMA-store epilogue, m = 37 / 100 its cluster reduction)."""
    a = torch.randn(m, k, generator=_seed(m)).to(dt)
    wg = (torch.randn(inter, k, generator=_seed(inter)) * 0.05).to(dt)
    wu = (torch.randn(inter, k, generator=_seed(inter + 1)) * 0.05).to(dt)
    cs = torch.rand(2, inter, generator=_seed(3)) + 0.5
    t, row_base, rows = (m + 2) // 3, 1, 4
    row_of = row_base + torch.arange(m) // t
    neurons = torch.tensor([5, -1, inter - 1], dtype=torch.int32)
    modes = torch.tensor([0, 1, 0], dtype=torch.int32)
    vals = torch.randn(3, rows, generator=_seed(4))
    gu = ops.interleave_gate_up(wg, wu)
    csi = ops.interleave_gate_up(cs[0][:, None], cs[1][:, None]).reshape(-1)
    out = ops.gemm_swiglu(a.cuda(), gu.cuda(), col_scale=csi.cuda(),
                          pushes=(neurons.cuda(), modes.cuda(), vals.cuda()), t=t, row_base=row_base)
    g = (a.float() @ wg.float().T) * cs[0]
    u = (a.float() @ wu.float().T) * cs[1]
    plist = [(None if n < 0 else n, "mul" if md else "add", vals[i])
             for i, (n, md) in enumerate(zip(neurons.tolist(), modes.tolist()))]
    ref = mixer.swiglu_push(torch.cat([g, u], 1), inter, plist, row_of)
    assert rel_max(out.float(), ref) < 1e-2
    assert ops.fault_status() == 0


def _q8_operand(q, s, group, dt):
    """The weight operand the tensor core sees and the factor on the f32 sum: 16-bit(f32(q) s) for group scales (the
    16-bit pack's value), q itself with the row scale on the sum for one scale per row."""
    k = q.shape[1]
    if group == k:
        return q.double(), s[:, 0].double()
    return (q.float() * s.repeat_interleave(group, 1)).to(dt).double(), torch.ones(q.shape[0], dtype=torch.float64)


@pytest.mark.parametrize("m,n,k,group,dt", [(9, 1000, 1024, 1024, torch.bfloat16), (40, 8224, 1024, 1024, torch.bfloat16),
                                            (130, 1024, 3584, 128, torch.bfloat16), (256, 8224, 1024, 128, torch.bfloat16),
                                            (256, 1024, 3584, 3584, torch.float16), (64, 384, 512, 64, torch.bfloat16)])
def test_q8_gemm(ops, m, n, k, group, dt):
    """int8 weights streamed into the decode GEMM and converted on chip (engine/kernels.js:97-151): store (f32 and
    16-bit) and residual add, against a float64 product of the same operands (f32 accumulation bounds the error)."""
    q = torch.randint(-127, 128, (n, k), generator=_seed(n), dtype=torch.int8)
    s = torch.rand(n, k // group, generator=_seed(k)) * 1e-2 + 1e-3
    x = torch.randn(m, k, generator=_seed(m)).to(dt)
    wop, post = _q8_operand(q, s, group, dt)
    ref = (x.double() @ wop.T) * post
    qd, sd, xd = q.cuda(), s.cuda(), x.cuda()
    y = ops.q8_gemm(xd, qd, sd, out_dtype=torch.float32)
    assert rel_max(y, ref) < 1e-5 * max(1.0, k / 1024)
    y16 = ops.q8_gemm(xd, qd, sd, out_dtype=dt)
    assert rel_max(y16.float(), ref) < 8e-3
    x0 = torch.randn(m, n, generator=_seed(2))
    acc = ops.q8_gemm(xd, qd, sd, y=x0.clone().cuda(), accumulate=True)
    assert rel_max(acc, x0.double() + ref) < 1e-5 * max(1.0, k / 1024)
    if dt == torch.bfloat16 and group == k:  # the 16-bit pack of the same weights through the bf16 GEMM
        yp = ops.gemm_bf16(xd, qd.to(torch.bfloat16), col_scale=sd[:, 0].contiguous(), out_dtype=torch.float32)
        assert rel_max(y, yp) < 1e-5 * max(1.0, k / 1024)
    assert ops.fault_status() == 0


@pytest.mark.parametrize("m,inter,k,group,dt", [(37, 128, 256, 128, torch.bfloat16), (256, 3584, 1024, 1024, torch.bfloat16),
                                                (100, 3584, 1024, 128, torch.float16), (200, 512, 256, 256, torch.bfloat16)])
def test_q8_gemm_swiglu(ops, m, inter, k, group, dt):
    """gate|up on int8 weights in their own row order [gate | up], read through the 16-bit pack's interleave, with
    SwiGLU fused (kernels_qwen35.js:250-280): against float64 on the same operands (16-bit output rounding)."""
    q = torch.randint(-127, 128, (2 * inter, k), generator=_seed(inter), dtype=torch.int8)
    s = torch.rand(2 * inter, k // group, generator=_seed(k + 1)) * 1e-2 + 1e-3
    x = torch.randn(m, k, generator=_seed(m + 3)).to(dt)
    wop, post = _q8_operand(q, s, group, dt)
    gu = (x.double() @ wop.T) * post
    g, u = gu[:, :inter], gu[:, inter:]
    ref = g / (1 + torch.exp(-g)) * u
    out = ops.q8_gemm(x.cuda(), q.cuda(), s.cuda(), swiglu=True)
    assert out.shape == (m, inter) and out.dtype == dt
    assert rel_max(out.float(), ref) < 1e-2
    assert ops.fault_status() == 0


def test_rmsnorm(ops):
    x = torch.randn(7, 1024, generator=_seed(9)) * 3
    w = torch.randn(1024, generator=_seed(10)) * 0.1
    y = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6)
    assert rel_max(y, mixer.rmsnorm(x, w, 1e-6)) < 1e-6
    yb = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6, out_dtype=torch.bfloat16)
    assert rel_max(yb.float(), mixer.rmsnorm(x, w, 1e-6)) < 8e-3


# ---------------------------------------------------------------------------------------------------------------
# Gated DeltaNet scan (kernels_qwen35.js:183-247; transformers torch_recurrent_gated_delta_rule)


def _gdn_inputs(b, t, h, seed, normed):
    g = _seed(seed)
    q = torch.randn(b, t, h, 128, generator=g)
    k = torch.randn(b, t, h, 128, generator=g)
    if normed:
        q, k = mixer.l2norm(q), mixer.l2norm(k)
    v = torch.randn(b, t, h, 128, generator=g)
    beta = torch.sigmoid(torch.randn(b, t, h, generator=g))
    gg = -torch.nn.functional.softplus(torch.randn(b, t, h, generator=g))
    s0 = torch.randn(b, h, 128, 128, generator=g) * 0.05
    return q, k, v, gg, beta, s0


@pytest.mark.parametrize("b,t,h", [(1, 1, 16), (2, 37, 4), (8, 3, 16), (40, 1, 16)])
def test_gdn_recurrent_f32(ops, b, t, h):
    q, k, v, g, beta, s0 = _gdn_inputs(b, t, h, b * 100 + t, False)
    ro, rs = mixer.recurrent_gated_delta_rule(q.double(), k.double(), v.double(), g.double(), beta.double(),
                                              state=s0.double())
    st = s0.clone().cuda()
    o = ops.gdn_recurrent(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), st, l2norm_qk=True)
    assert rel_max(o, ro) < 1e-4
    assert rel_max(st, rs) < 1e-4


def test_gdn_recurrent_steps_equal_one_call(ops):
    q, k, v, g, beta, s0 = _gdn_inputs(2, 6, 4, 77, True)
    st1 = s0.clone().cuda()
    o1 = ops.gdn_recurrent(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), st1, l2norm_qk=False)
    st2 = s0.clone().cuda()
    outs = []
    for i in range(6):
        sl = lambda x: x[:, i:i + 1].contiguous().cuda()
        outs.append(ops.gdn_recurrent(sl(q), sl(k), sl(v), sl(g), sl(beta), st2, l2norm_qk=False))
    assert rel_max(torch.cat(outs, 1), o1) < 1e-6
    assert rel_max(st2, st1) < 1e-6


def test_gdn_recurrent_bf16(ops):
    q, k, v, g, beta, s0 = _gdn_inputs(2, 40, 16, 5, True)
    qb, kb, vb = (x.to(torch.bfloat16) for x in (q, k, v))
    ro, rs = mixer.recurrent_gated_delta_rule(qb.double(), kb.double(), vb.double(), g.double(), beta.double(),
                                              state=s0.double(), l2norm_qk=False)
    st = s0.clone().cuda()
    o = ops.gdn_recurrent(qb.cuda(), kb.cuda(), vb.cuda(), g.cuda(), beta.cuda(), st, l2norm_qk=False)
    assert rel_max(o.float(), ro) < 2e-2
    assert rel_max(st, rs) < 1e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,t,h,l2", [(1, 64, 2, False), (2, 100, 4, True), (1, 300, 16, False), (3, 17, 2, True),
                                      (2, 1024, 16, False), (4, 2, 16, False), (3, 5, 4, True), (216, 16, 16, False)])
def test_gdn_chunk_16bit(ops, dtype, b, t, h, l2):
    """Chunked tensor-core scan vs the oracle's chunk rule (f64) on the same 16-bit inputs; 16-bit bound 2e-2."""
    q, k, v, g, beta, s0 = _gdn_inputs(b, t, h, 1000 + t, not l2)
    qb, kb, vb = (x.to(dtype) for x in (q, k, v))
    ro, rs = mixer.chunk_gated_delta_rule(qb.double(), kb.double(), vb.double(), g.double(), beta.double(),
                                          state=s0.double(), l2norm_qk=l2)
    st = s0.clone().cuda()
    o = ops.gdn_chunk(qb.cuda(), kb.cuda(), vb.cuda(), g.cuda(), beta.cuda(), st, l2norm_qk=l2)
    assert rel_max(o.float(), ro) < 2e-2
    assert rel_max(st, rs) < 2e-2


def test_gdn_chunk_matches_recurrent_kernel(ops):
    """The two GPU forms of the scan agree (f32 inputs; the chunk kernel rounds its operands to bf16)."""
    q, k, v, g, beta, s0 = _gdn_inputs(2, 200, 16, 4242, True)
    st1, st2 = s0.clone().cuda(), s0.clone().cuda()
    o1 = ops.gdn_recurrent(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), st1, l2norm_qk=False)
    o2 = ops.gdn_chunk(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), st2, l2norm_qk=False)
    assert rel_max(o2, o1) < 2e-2
    assert rel_max(st2, st1) < 2e-2


# ---------------------------------------------------------------------------------------------------------------
# attention (kernels_qwen35.js:73-123; transformers eager attention with repeat_kv, sigmoid gate)


def _attn_ref(q, kc, vc, start, gate):
    b, t, nh, hd = q.shape
    out = torch.zeros(b, t, nh, hd, dtype=torch.float64)
    for r in range(b):
        n_keys = [int(start[r]) + i + 1 for i in range(t)]
        out[r] = mixer.cached_attention(q[r].double(), kc[r].double(), vc[r].double(), n_keys, 1 / math.sqrt(hd))
    if gate is not None:
        out = out * torch.sigmoid(gate.double())
    return out


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2), (torch.float16, 2e-2)])
@pytest.mark.parametrize("b,t,starts,max_len,nh,nkv", [(2, 70, [0, 30], 128, 8, 2), (3, 1, [0, 5, 900], 1024, 8, 2),
                                                        (2, 1, [4095, 3000], 4096, 8, 2), (1, 33, [100], 256, 8, 2),
                                                        (1, 300, [0], 512, 8, 2), (2, 129, [7, 0], 200, 4, 2),
                                                        (1, 65, [3], 128, 2, 2)])
def test_attention(ops, dtype, tol, b, t, starts, max_len, nh, nkv):
    g = _seed(b * 1000 + t)
    hd = 256
    q = torch.randn(b, t, nh, hd, generator=g).to(dtype)
    kc = torch.randn(b, max_len, nkv, hd, generator=g).to(dtype)
    vc = torch.randn(b, max_len, nkv, hd, generator=g).to(dtype)
    gate = torch.randn(b, t, nh, hd, generator=g).to(dtype)
    start = torch.tensor(starts, dtype=torch.int32)
    ref = _attn_ref(q.float(), kc.float(), vc.float(), start, gate.float())
    o = ops.attention(q.cuda(), kc.cuda(), vc.cuda(), start.cuda(), gate=gate.cuda())
    assert rel_max(o.float(), ref) < tol


# ---------------------------------------------------------------------------------------------------------------
# DeltaNet conv prologue (kernels_qwen35.js:129-178, 208-229): causal conv + SiLU + q/k l2norm + gates, state carried
# across calls.  Call sequences mix the register-staged kernel (f32, or fewer than 64 token rows) and the TMA-fed one
# (16-bit, >= 64 token rows), several 64-token tiles per block and several blocks per row (> 512 tokens), and token
# counts whose last tile has an odd number of tokens modulo 16 (37, 3, 129).


def _conv_ref(y, conv_w, state, a_log, dt_bias, hk, hv):
    b, t, _ = y.shape
    kd, vd = hk * 128, hv * 128
    cd = 2 * kd + vd
    out, new_state = mixer.causal_conv1d(y[..., :cd].float(), conv_w, state)
    q = mixer.l2norm(out[..., :kd].reshape(b, t, hk, 128)).reshape(b, t, kd)
    k = mixer.l2norm(out[..., kd:2 * kd].reshape(b, t, hk, 128)).reshape(b, t, kd)
    beta, g = mixer.gdn_gates(y[..., cd + vd + hv:cd + vd + 2 * hv].float(), y[..., cd + vd:cd + vd + hv].float(),
                              a_log, dt_bias)
    return torch.cat([q, k, out[..., 2 * kd:]], -1), g, beta, new_state


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2), (torch.float16, 2e-3)])
@pytest.mark.parametrize("b,calls,hk,hv", [(2, [700, 3, 37, 1, 2], 4, 4), (1, [1100], 16, 16),
                                           (3, [17, 64, 129], 2, 4), (8, [37], 16, 16)])
def test_gdn_conv(ops, dtype, tol, b, calls, hk, hv):
    gen = _seed(sum(calls) + 31 * b + hk)
    cd = 2 * hk * 128 + hv * 128
    w = cd + hv * 128 + 2 * hv
    conv_w = torch.randn(cd, 4, generator=gen) * 0.3
    a_log = torch.empty(hv).uniform_(0, 16, generator=gen).log()
    dt_bias = torch.ones(hv)
    state = torch.randn(b, 3, cd, generator=gen) * 0.5
    st_gpu = state.clone().cuda()
    for t in calls:
        y = torch.randn(b, t, w, generator=gen).to(dtype)
        qkv, g, beta = ops.gdn_conv(y.cuda(), conv_w.cuda(), st_gpu, a_log.cuda(), dt_bias.cuda(), hk, hv)
        rq, rg, rb, state = _conv_ref(y, conv_w, state, a_log, dt_bias, hk, hv)
        assert rel_max(qkv.float(), rq) < tol, t
        assert rel_max(g, rg) < 1e-5 and rel_max(beta, rb) < 1e-5, t
        assert torch.equal(st_gpu.cpu(), state.float()), t  # the carried inputs, exactly
    assert ops.fault_status() == 0


# ---------------------------------------------------------------------------------------------------------------
# config 2's chunked-scan shapes (B in {1, 8}, T in {512, 4096, 16384}, H = 16, chunk 64, bf16 inputs, f32 state),
# checked against the oracle's chunk rule on three of the sixteen heads (the CPU cost of all heads is large)


@pytest.mark.parametrize("b,t", [(1, 512), (8, 512), (1, 4096), (8, 4096), (1, 16384), (8, 16384)])
def test_gdn_chunk_config2_shapes(ops, b, t):
    h, heads = 16, [0, 9, 15]
    gen = torch.Generator(device="cuda").manual_seed(b * 100003 + t)
    rn = lambda *s: torch.randn(*s, generator=gen, device="cuda")
    q, k = mixer.l2norm(rn(b, t, h, 128)), mixer.l2norm(rn(b, t, h, 128))
    v = rn(b, t, h, 128)
    beta = torch.sigmoid(rn(b, t, h))
    g = -torch.nn.functional.softplus(rn(b, t, h))
    qb, kb, vb = (x.to(torch.bfloat16).contiguous() for x in (q, k, v))
    st = torch.zeros(b, h, 128, 128, device="cuda")
    o = ops.gdn_chunk(qb, kb, vb, g.contiguous(), beta.contiguous(), st, l2norm_qk=False)
    sl = lambda x: x[:, :, heads].float().cpu()
    ro, rs = mixer.chunk_gated_delta_rule(sl(qb), sl(kb), sl(vb), sl(g), sl(beta), state=None, l2norm_qk=False)
    assert rel_max(o[:, :, heads].float(), ro) < 2e-2
    assert rel_max(st[:, heads], rs) < 2e-2
    assert not torch.isnan(o.float()).any()
    assert ops.fault_status() == 0


# ---------------------------------------------------------------------------------------------------------------
# config 3's attention shapes: prefill at B = 4, T in {1024, 4096, 16384} (8 q / 2 kv heads, hd 256, sigmoid gate)
# checked on sampled query positions; decode at B = 32 against an 8192-token cache, checked in full


@pytest.mark.parametrize("t", [1024, 4096, 16384])
def test_attention_prefill_config3(ops, t):
    b, nh, nkv, hd = 4, 8, 2, 256
    gen = torch.Generator(device="cuda").manual_seed(t)
    rn = lambda *s: torch.randn(*s, generator=gen, device="cuda").to(torch.bfloat16)
    q, gate = rn(b, t, nh, hd), rn(b, t, nh, hd)
    kc, vc = rn(b, t, nkv, hd), rn(b, t, nkv, hd)
    start = torch.zeros(b, dtype=torch.int32, device="cuda")
    o = ops.attention(q, kc, vc, start, gate=gate)
    pos = sorted(set([0, 1, 63, 64, 127, 128, t // 2, t - 65, t - 2, t - 1] +
                     torch.randint(0, t, (6,), generator=_seed(t)).tolist()))
    kf, vf = kc.float().cpu(), vc.float().cpu()
    for r in range(b):
        qs = q[r, pos].float().cpu()
        ref = torch.stack([mixer.cached_attention(qs[i:i + 1], kf[r], vf[r], [p + 1], hd ** -0.5)[0]
                           for i, p in enumerate(pos)])
        ref = ref * torch.sigmoid(gate[r, pos].float().cpu())
        assert rel_max(o[r, pos].float(), ref) < 2e-2, r
    assert not torch.isnan(o.float()).any()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ragged", [False, True])
def test_attention_decode_config3(ops, dtype, ragged):
    b, nh, nkv, hd, max_len = 32, 8, 2, 256, 8192
    gen = torch.Generator(device="cuda").manual_seed(32 + ragged)
    rn = lambda *s: torch.randn(*s, generator=gen, device="cuda").to(dtype)
    q, gate = rn(b, 1, nh, hd), rn(b, 1, nh, hd)
    kc, vc = rn(b, max_len, nkv, hd), rn(b, max_len, nkv, hd)
    starts = (torch.randint(0, max_len, (b,), generator=_seed(5)) if ragged else torch.full((b,), max_len - 1))
    starts[0] = max_len - 1
    start = starts.to(torch.int32).cuda()
    o = ops.attention(q, kc, vc, start, gate=gate)
    ref = _attn_ref(q.float().cpu(), kc.float().cpu(), vc.float().cpu(), starts, gate.float().cpu())
    assert rel_max(o.float(), ref) < 2e-2


# ---------------------------------------------------------------------------------------------------------------
# push-probe statistics (engine/analysis.js:480-537): lse, target mass and weighted target lse per row; KL, dp, gain
# and the per-vocabulary delta against each row's unsteered row


@pytest.mark.parametrize("n,vocab", [(6, 248320), (9, 1001), (216, 248320)])
def test_push_stats(ops, n, vocab):
    from oracle import probe
    gen = _seed(n + vocab)
    logits = torch.randn(n, vocab, generator=gen) * 3
    # triples (+, 0, -) of one context: the middle row is the base of the other two
    base = torch.tensor([(r // 3) * 3 + 1 if r % 3 != 1 else -1 for r in range(n)], dtype=torch.int32)
    for r in range(n):
        if r % 3 != 1:  # a steered row: its logits move away from the base a little
            logits[r] = logits[(r // 3) * 3 + 1] + torch.randn(vocab, generator=gen) * 0.3
    targets = torch.randint(0, vocab, (64,), generator=gen, dtype=torch.int32)
    targets[5] = vocab + 3  # an out-of-range id counts as probability 0
    logw = torch.log(torch.rand(64, generator=gen) + 0.1)
    d0 = torch.randn(n, vocab, generator=gen)
    stats, d = ops.push_stats(logits.cuda(), base.cuda(), targets.cuda(), logw.cuda(), d=d0.clone().cuda())
    rs, rd = probe.push_stats(logits.numpy(), base.numpy(), targets.numpy(), logw.numpy())
    st = stats.double().cpu().numpy()
    for c in range(6):
        err = np.abs(st[:, c] - rs[:, c])
        assert (err <= 1e-5 + 1e-4 * np.abs(rs[:, c])).all(), (c, err.max())
    assert rel_max(d, torch.from_numpy(rd) + d0.double()) < 1e-5
    assert ops.fault_status() == 0
