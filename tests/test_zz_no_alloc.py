"""duo_attention_noalloc, the attention entry point for callers that cannot allocate device memory (a serving stack
whose pooled allocator owns it all, or a decode loop where cudaMalloc's implicit synchronisation is not allowed).

It keeps its split-K decode partials in a fixed static device array instead of a workspace the library allocates.
These tests call it through the C ABI and compare it with duo_attention on the same inputs (bf16 tolerance 2e-2 of
the other GPU tests, and in practice bit for bit: same kernels, same split plan), on two calls in a row with
different shapes so that stale contents of the shared array would show.  This file sorts last so that a run that
stops at the first failure has already run every other test; it passes alone in a fresh process as well."""
import ctypes as C

import pytest
import torch

from conftest import rel_max

pytestmark = pytest.mark.gpu


def _inputs(b, max_len, starts, seed, nh=8, nkv=2, hd=256, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to(dtype).cuda()
    q, gate = mk(b, 1, nh, hd), mk(b, 1, nh, hd)
    kc, vc = mk(b, max_len, nkv, hd), mk(b, max_len, nkv, hd)
    return q, kc, vc, torch.tensor(starts, dtype=torch.int32).cuda(), gate


def _call(name, q, kc, vc, start, gate):
    from duo import lib as L
    b, t, nh, hd = q.shape
    _, max_len, nkv, _ = kc.shape
    o = torch.full_like(q, float("nan"))
    code = {torch.float32: L.DUO_F32, torch.bfloat16: L.DUO_BF16, torch.float16: L.DUO_F16}[q.dtype]
    st = L.lib().__getattr__(name)(L.ptr(q), L.ptr(kc), L.ptr(vc), L.ptr(start), L.ptr(gate), nh * hd, L.ptr(o),
                                   code, b, t, nh, nkv, hd, max_len, C.c_float(hd ** -0.5),
                                   L.stream_ptr())
    return st, o


# bf16 and f16 take the tensor-core decode kernel and its split plan, f32 the CUDA-core kernel and its own plan: the
# scratch size the entry point checks must follow each of them
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_noalloc_matches_allocating_entry_point_twice(cuda, dtype):
    from duo import lib as L
    cases = [(4, 4096, [4095, 17, 2048, 3000], 1), (2, 2048, [2047, 100], 2)]
    for b, max_len, starts, seed in cases:  # two calls in a row on the shared static scratch
        q, kc, vc, start, gate = _inputs(b, max_len, starts, seed, dtype=dtype)
        st, o_na = _call("duo_attention_noalloc", q, kc, vc, start, gate)
        assert st == L.DUO_OK, L.lib().duo_last_error()
        st, o_ref = _call("duo_attention", q, kc, vc, start, gate)
        assert st == L.DUO_OK, L.lib().duo_last_error()
        torch.cuda.synchronize()
        assert not torch.isnan(o_na.float()).any()
        assert rel_max(o_na.float(), o_ref.float()) < 2e-2
        assert torch.equal(o_na, o_ref)


def test_noalloc_rejects_a_call_larger_than_its_scratch(cuda):
    from duo import lib as L
    # 64 rows x 8 heads x 3 splits x 258 floats = 396,288 > 262,144: refused before any launch
    q, kc, vc, start, gate = _inputs(64, 8192, [8191] * 64, 3)
    st, o = _call("duo_attention_noalloc", q, kc, vc, start, gate)
    assert st == L.DUO_EINVAL
    assert b"static array holds" in L.lib().duo_last_error()
    torch.cuda.synchronize()
    assert torch.isnan(o.float()).all()  # nothing ran
