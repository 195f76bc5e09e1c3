"""GPU: index lists read from device memory are range-checked in the kernels.

A bad host-side index (one past the end, negative) must become an error code
in the status word, never an out-of-bounds device access: the quantiser's
fused gather, the row gather and the dequantiser each get the source length
and redirect an out-of-range index to element 0 after flagging AKV_ERR_SHAPE
(like the paged decode's block-table check in test_gpu_paged.py).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
AKV_ERR_SHAPE = -1


def _status():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("bad", [50, -1, 1 << 40])
def test_gather_rows_out_of_range_sets_status(bad):
    from akv import tiering
    x = torch.randn(2, 3, 50, 128, device=DEV).half()
    st = _status()
    idx = torch.tensor([0, 7, bad, 3], device=DEV)
    y = tiering.gather_rows(x, idx, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == AKV_ERR_SHAPE
    good = [0, 1, 3]
    torch.testing.assert_close(y[:, :, good], x[:, :, idx[good]], rtol=0, atol=0)
    torch.testing.assert_close(y[:, :, 2], x[:, :, 0], rtol=0, atol=0)  # redirected to row 0
    # in-range indices leave the status untouched
    st2 = _status()
    tiering.gather_rows(x, torch.tensor([49, 0], device=DEV), status=st2)
    torch.cuda.synchronize()
    assert int(st2.item()) == 0


def test_quantize_gather_out_of_range_sets_status():
    import akv
    g = torch.Generator(device=DEV).manual_seed(3)
    k = torch.randn(1, 2, 40, 128, generator=g, device=DEV).half()
    v = torch.randn(1, 2, 40, 128, generator=g, device=DEV).half()
    arena = akv.WarmArena(1, 2, 128, 4, 2, max_blocks=4, device=DEV)
    st = _status()
    idx = torch.tensor([[1, 5, 40, 9]], device=DEV)  # 40 is one past the last row
    arena.append(k, v, tok_idx=idx, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == AKV_ERR_SHAPE
    st2 = _status()
    arena.append(k, v, tok_idx=torch.tensor([[0, 39]], device=DEV), status=st2)
    torch.cuda.synchronize()
    assert int(st2.item()) == 0


def test_dequantize_out_of_range_sets_status():
    import akv
    g = torch.Generator(device=DEV).manual_seed(4)
    k = torch.randn(1, 2, 64, 128, generator=g, device=DEV).half()
    arena = akv.WarmArena(1, 2, 128, 3, 3, max_blocks=4, device=DEV)
    arena.append(k, k)
    st = _status()
    dk, _ = arena.dequantize(tok_idx=torch.tensor([3, 64], device=DEV), status=st)  # 2 blocks = slots 0..63
    torch.cuda.synchronize()
    assert int(st.item()) == AKV_ERR_SHAPE
    assert torch.isfinite(dk.float()).all()
    ref, _ = arena.dequantize(tok_idx=torch.tensor([3, 0], device=DEV))
    torch.testing.assert_close(dk, ref, rtol=0, atol=0)
