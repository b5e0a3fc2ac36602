"""GPU tests of the engine calls around the GEMV: greedy pick, graph capture,
the tile repack, async copies."""

from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod(cuda_lib):
    import torch
    torch.cuda.set_device(0)
    return torch


@pytest.fixture(scope="module")
def eng(pkg, torch_mod):
    e = pkg.Engine(0)
    yield e
    e.close()


def _pick(torch, eng, y_np, base=0):
    y = torch.from_numpy(y_np.astype(np.float32)).cuda()
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    eng.argmax(y, y.numel(), out, index_base=base)
    eng.sync()
    o = out.cpu().numpy()
    return int(o[0]), float(o[1:2].view(np.float32)[0])


def _scan(y):
    """tp_llama.cpp:879-882."""
    best = 0
    for i in range(1, len(y)):
        if y[i] > y[best]:
            best = i
    return best


@pytest.mark.parametrize("n", [1, 7, 512, 4097, 16032, 128256])
def test_argmax_matches_the_runtime_scan(torch_mod, eng, n):
    rng = np.random.default_rng(n)
    y = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        y[n // 3] = y[n // 2] = y.max() + 1.0      # a tie: the lower index wins
    i, v = _pick(torch_mod, eng, y, base=5)
    assert i - 5 == int(np.argmax(y)) == _scan(y) and v == y.max()


def test_argmax_nan_rules(torch_mod, eng):
    y = np.array([np.nan, 1.0, 5.0, 2.0], np.float32)
    assert _pick(torch_mod, eng, y)[0] == _scan(y) == 0          # NaN first: never beaten
    y = np.array([1.0, np.nan, 5.0, np.nan, 5.0], np.float32)
    assert _pick(torch_mod, eng, y)[0] == _scan(y) == 2          # NaN later: never wins
    y = np.full(100, -np.inf, np.float32)
    assert _pick(torch_mod, eng, y)[0] == _scan(y) == 0


def test_graph_replay_matches_eager_calls(torch_mod, pkg, oracle):
    """A captured chain of engine calls replays to the same bits as the calls run one by one."""
    torch = torch_mod
    stream = torch.cuda.Stream()
    e = pkg.Engine(0, stream=stream.cuda_stream)
    blocks1 = oracle.quantize_q4_0(cases.std_weights(512, 1024, 91))
    blocks2 = oracle.quantize_q4_0(cases.std_weights(1024, 512, 92))
    W1 = e.repack(pkg.QMat(torch.from_numpy(blocks1.reshape(-1).copy()).cuda(), 512, 1024))
    W2 = e.repack(pkg.QMat(torch.from_numpy(blocks2.reshape(-1).copy()).cuda(), 1024, 512))
    x = torch.from_numpy(cases.std_weights(1, 1024, 93)[0]).cuda()
    y1 = torch.empty(512, device="cuda")
    y2 = torch.empty(1024, device="cuda")
    sel = torch.zeros(2, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()

    def chain():
        e.gemv_f32(W1, x, y1)
        e.gemv_f32(W2, y1, y2)
        e.argmax(y2, 1024, sel)

    chain()
    e.sync()
    want_y2, want_sel = y2.cpu().numpy().copy(), sel.cpu().numpy().copy()
    y1_cpu = oracle.gemv_q4_0_f32(blocks1, 1024, x.cpu().numpy())
    assert np.array_equal(y1.cpu().numpy().view(np.uint32), y1_cpu.view(np.uint32))
    assert np.array_equal(want_y2.view(np.uint32), oracle.gemv_q4_0_f32(blocks2, 512, y1_cpu).view(np.uint32))
    e.capture_begin()
    chain()
    g = e.capture_end()
    y2.zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        g.launch()
    e.sync()
    assert np.array_equal(y2.cpu().numpy().view(np.uint32), want_y2.view(np.uint32))
    assert np.array_equal(sel.cpu().numpy(), want_sel)
    host = torch.zeros(1024).pin_memory()
    e.copy_async(int(host.data_ptr()), int(y2.data_ptr()), 4096)
    e.sync()
    assert np.array_equal(host.numpy().view(np.uint32), want_y2.view(np.uint32))
    g.close()
    e.close()


@pytest.mark.parametrize("rows", [1, 17, 2048, 16032])
@pytest.mark.parametrize("fuse", [0, 1])
def test_fused_greedy_pick_matches_gemv_then_scan(torch_mod, pkg, eng, oracle, rows, fuse):
    """lm_head GEMV with the pick fused in: y bit-exact, pick = the runtime's scan of y."""
    torch = torch_mod
    k = 2048
    w = cases.std_weights(rows, k, 300 + rows)
    if rows > 40:
        w[rows // 2] = w[rows // 3]            # two equal rows: equal logits, the lower index wins
    blocks = oracle.quantize_q4_0(w)
    x = cases.std_weights(1, k, 301)[0]
    want = oracle.gemv_q4_0_f32(blocks, k, x)
    W = eng.repack(pkg.QMat(torch.from_numpy(blocks.reshape(-1).copy()).cuda(), rows, k))
    eng.configure(fuse_quantize=fuse)
    y = torch.empty(rows, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    for _ in range(3):                          # the ticket resets itself between calls
        eng.gemv_argmax_f32(W, torch.from_numpy(x).cuda(), y, out, index_base=1000)
        eng.sync()
        o = out.cpu().numpy()
        assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
        assert int(o[0]) - 1000 == _scan(want)
        assert o[1:2].view(np.float32)[0] == want[_scan(want)]
    eng.configure(fuse_quantize=0)
