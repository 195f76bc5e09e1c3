"""GPU: DecodeGraph captures a multi-layer decode step (with pinned-host
uploads and downloads on forked streams) and replays it bit-identically to
eager issue; new query values written into the captured buffers are picked
up by the next replay."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _layers(g, L, B=2, Hq=8, Hkv=2, D=128, n_warm=32 * 9 + 5, n_hot=70):
    import akv
    out = []
    for _ in range(L):
        a = akv.WarmArena(B, Hkv, D, 4, 2, outlier_fraction=0.01, max_blocks=(n_warm + 31) // 32, device=DEV)
        a.append(torch.randn(B, Hkv, n_warm, D, generator=g, device=DEV).half(),
                 torch.randn(B, Hkv, n_warm, D, generator=g, device=DEV).half(), group=32)
        hk = torch.randn(B, Hkv, n_hot, D, generator=g, device=DEV).half()
        hv = torch.randn(B, Hkv, n_hot, D, generator=g, device=DEV).half()
        out.append((a, hk, hv))
    return out


def test_decode_graph_matches_eager_and_tracks_inputs():
    import akv
    g = torch.Generator(device=DEV).manual_seed(0)
    L, B, Hq, D = 3, 2, 8, 128
    layers = _layers(g, L)
    q_host = torch.randn(L, B, Hq, D, generator=torch.Generator().manual_seed(1)).half().pin_memory()
    o_host = torch.empty(L, B, Hq, D, dtype=torch.float16).pin_memory()
    q_dev = torch.empty(L, B, Hq, D, dtype=torch.float16, device=DEV)
    o_dev = torch.empty_like(q_dev)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def step():
        cur = torch.cuda.current_stream()
        s_in.wait_stream(cur)
        with torch.cuda.stream(s_in):
            q_dev.copy_(q_host, non_blocking=True)
        cur.wait_stream(s_in)
        for l, (a, hk, hv) in enumerate(layers):
            akv.mixed_tier_decode_attention(q_dev[l], hk, hv, a, out=o_dev[l])
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_out):
            o_host.copy_(o_dev, non_blocking=True)
        cur.wait_stream(s_out)

    step()
    torch.cuda.synchronize()
    eager = o_host.clone()
    try:
        dg = akv.DecodeGraph(step)
    except RuntimeError as exc:  # capture of pinned-host copies refused by this torch build
        pytest.skip(f"capture refused: {exc}")
    o_host.zero_()
    dg.replay()
    torch.cuda.synchronize()
    assert torch.equal(o_host, eager)
    # new queries in the captured pinned buffer: the replay decodes them
    q_host.copy_(torch.randn(L, B, Hq, D, generator=torch.Generator().manual_seed(2)).half())
    step()
    torch.cuda.synchronize()
    eager2 = o_host.clone()
    o_host.zero_()
    dg.replay()
    torch.cuda.synchronize()
    assert torch.equal(o_host, eager2) and not torch.equal(eager2, eager)
    dg.reset()
