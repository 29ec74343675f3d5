"""Host-side layout helpers of the decode GEMM and the fp8 scales (CPU only)."""

import pytest

torch = pytest.importorskip("torch")


def test_gate_up_interleave_round_trip():
    from sparknet.ops.decode_gemm import INTERLEAVE_ROWS, interleave_gate_up, split_gate_up

    F, K = 3 * INTERLEAVE_ROWS, 40
    gate = torch.arange(F * K, dtype=torch.float32).view(F, K)
    up = -gate
    w = interleave_gate_up(gate, up)
    assert w.shape == (2 * F, K)
    # 128-row tile t = [gate rows 64t..64t+63 ; up rows 64t..64t+63]
    for t in range(F // INTERLEAVE_ROWS):
        assert torch.equal(w[128 * t:128 * t + 64], gate[64 * t:64 * t + 64])
        assert torch.equal(w[128 * t + 64:128 * t + 128], up[64 * t:64 * t + 64])
    g2, u2 = split_gate_up(w)
    assert torch.equal(g2, gate) and torch.equal(u2, up)
    with pytest.raises(ValueError):
        interleave_gate_up(gate[:10], up[:10])


def test_fp8_scale_chunk_layout_decodes():
    """Byte (row, 128-column block) of the tcgen05.cp chunk layout: chunk (rb, kb) of
    512 bytes, row 32*g + i at byte 16*i + 4*g (+ j for the K step)."""
    from sparknet.ops import fp8

    rows, k = 200, 384
    kb = k // 128
    sf = torch.zeros(fp8.scale_bytes(rows, k), dtype=torch.uint8)
    want = torch.zeros(rows, kb, dtype=torch.int64)
    for r in range(rows):
        for b in range(kb):
            e = 100 + (r * 7 + b * 3) % 60
            want[r, b] = e
            rb, rr = divmod(r, 128)
            off = (rb * kb + b) * 512 + (rr % 32) * 16 + (rr // 32) * 4
            sf[off:off + 4] = e
    assert torch.equal(fp8.scale_exponents(sf, rows, k).to(torch.int64), want)
    dense = fp8.scales_to_dense(sf, rows, k)
    assert torch.equal(dense, torch.ldexp(torch.ones(rows, kb), (want - 127).to(torch.int32)))
    assert fp8.scale_bytes(128, 128) == 512 and fp8.scale_bytes(129, 256) == 2 * 2 * 512
