"""K13 data-movement kernels on one GPU: the store and load paths move bytes exactly
(local addresses stand in for a peer's mapping; the kernels only see addresses)."""

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("nbytes,blocks,threads,ppt", [(16, 1, 32, 1), (10240, 8, 512, 1), (491520, 37, 256, 4),
                                                      (4 << 20, 148, 512, 8)])
def test_nvlink_move_copies_exactly(device, native, mode, nbytes, blocks, threads, ppt):
    src = torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device=device)
    dst = torch.zeros(nbytes + 64, dtype=torch.uint8, device=device)
    native.nvlink_move(src.data_ptr(), dst.data_ptr(), nbytes, mode, blocks, threads, ppt, device.index or 0)
    torch.cuda.synchronize()
    assert torch.equal(dst[:nbytes], src)
    assert not dst[nbytes:].any(), "wrote past the end"


def test_nvlink_move_rejects_misaligned(device, native):
    src = torch.zeros(64, dtype=torch.uint8, device=device)
    with pytest.raises(ValueError):
        native.nvlink_move(src.data_ptr(), src.data_ptr() + 32, 24, 0, 1, 32, 1, device.index or 0)
    with pytest.raises(ValueError):
        native.nvlink_move(src.data_ptr(), src.data_ptr() + 32, 16, 0, 1, 48, 1, device.index or 0)
