"""The allocation-free decode-attention entry point (GPU).

Some callers cannot allocate device memory when they run attention: engines that have
already reserved the GPU's memory for their own pool, C hosts without a caching
allocator.  The library exports
``sparknet_decode_attention_noalloc``, whose scratch is a fixed array inside the
library.  This test calls that exported C symbol directly (ctypes), twice in a row,
and checks each result bit for bit against the allocating entry point on the same
inputs (the same kernel with the same split, so the same bits), and both against an
fp32 attention computed by torch.  It lives in its own file, collected last, so a
stopping run has run everything else first; it passes alone in a fresh process too.
"""

import ctypes
import math

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def load_symbols():
    from sparknet import _native

    native = _native.load()
    lib = ctypes.CDLL(native.__file__)
    fn = lib.sparknet_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    err = lib.sparknet_noalloc_last_error
    err.restype = ctypes.c_char_p
    need = lib.sparknet_decode_attention_scratch_bytes
    need.restype = ctypes.c_size_t
    need.argtypes = [ctypes.c_int] * 4
    return native, fn, err, need


def attention_fp32(q, k, v, lengths, scale):
    """Softmax attention of one query token per sequence over its first lengths[b] keys,
    in fp32 (grouped-query: query head h reads KV head h // (Hq / Hkv))."""
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(lengths[b])
        kb = k[b, :n].float().repeat_interleave(Hq // Hkv, dim=1)  # [n, Hq, D]
        vb = v[b, :n].float().repeat_interleave(Hq // Hkv, dim=1)
        scores = torch.einsum("hd,nhd->hn", q[b].float(), kb) * scale
        out[b] = torch.einsum("hn,nhd->hd", torch.softmax(scores, dim=-1), vb)
    return out


def test_noalloc_attention_matches_allocating_entry_point(device):
    native, fn, err, need = load_symbols()
    B, Hq, Hkv, L = 8, 64, 8, 1100
    Lmax = 1280
    scale = 1.0 / math.sqrt(128)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    stream = torch.cuda.current_stream(device).cuda_stream
    for call in range(2):  # two calls in a row share the scratch
        g = torch.Generator(device=device).manual_seed(40 + call)
        q = torch.randn(B, Hq, 128, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(B, Lmax, Hkv, 128, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(B, Lmax, Hkv, 128, generator=g, device=device).to(torch.bfloat16)
        lengths = torch.randint(1, L + 1, (B,), dtype=torch.int32, device=device, generator=g)
        ws = torch.zeros(native.attention_workspace_floats(B, Hq, Hkv, L, sms), dtype=torch.float32, device=device)
        want = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=device)
        native.decode_attention(q, k, v, lengths, want, ws, L, scale)
        got = torch.full_like(want, float("nan"))
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), lengths.data_ptr(), got.data_ptr(), B, Hq, Hkv, Lmax, L,
                scale, stream)
        assert rc == 0, err().decode()
        torch.cuda.synchronize(device)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), "differs from the allocating entry point"
        oracle = attention_fp32(q, k, v, lengths, scale)
        torch.testing.assert_close(got.float(), oracle, rtol=1e-2, atol=1e-2)
    assert 0 < need(B, Hq, Hkv, L) <= 8 << 20


def test_noalloc_rejects_problems_beyond_its_scratch(device):
    native, fn, err, need = load_symbols()
    B, Hq, Hkv, L = 256, 128, 8, 8192   # far more partials than the built-in scratch holds
    q = torch.zeros(1, dtype=torch.bfloat16, device=device)
    rc = fn(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), B, Hq, Hkv, L, L, 0.1,
            torch.cuda.current_stream(device).cuda_stream)
    assert rc == 2 and b"scratch" in err()
    assert need(B, Hq, Hkv, L) > 8 << 20
    rc = fn(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 1, 6, 4, 8, 8, 0.1,
            torch.cuda.current_stream(device).cuda_stream)
    assert rc == 1 and err()
