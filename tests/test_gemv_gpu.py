"""GPU parity: the sm_100a GEMV against the oracle and the reference's fixtures.

Every comparison is bit-exact (float32 bit patterns), because the contract
(src/llm_kv260/q4_0.py) pins every rounding. The inputs are the seeded ones of
tests/golden/cases.py; the expected digests came from the reference itself.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _y(hexstr: str) -> np.ndarray:
    return np.frombuffer(bytes.fromhex(hexstr), dtype=np.float32)


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


def _dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(np.uint8).copy()).cuda()


def _run_engine(torch, pkg, eng, blocks, k, x, fuse=0, packed=False, oracle=None, layout=1, **cfg):
    n = blocks.shape[0]
    W = pkg.QMat(_dev(torch, blocks), n, k)
    if layout == pkg.LAYOUT_TILES:
        W = eng.repack(W)
    y = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
    eng.configure(fuse_quantize=fuse, **cfg)
    if packed:
        xq, xd = oracle.quantize_q8_0(x)
        xp = _dev(torch, oracle.pack_x_for_engine(xq, xd))
        eng.gemv_q8(W, xp, y)
    else:
        eng.gemv_f32(W, torch.from_numpy(x).cuda(), y)
    eng.sync()
    out = y.cpu().numpy()
    eng.configure(fuse_quantize=0, stage_bytes=16384, stages=4, ctas_per_sm=2, xreg_chunks=8, kslices=1)
    return out


# ------------------------------------------------------------ golden pins

@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("fuse", [0, 1])
def test_golden_vector_on_gpu(torch_mod, pkg, eng, oracle, fuse, layout):
    """The reference's frozen digest (tests/test_q4_0_contract.py:181-191)."""
    blocks = oracle.quantize_q4_0(cases.std_weights(96, 2048, 2024))
    x = cases.std_weights(1, 2048, 2025)[0]
    y = _run_engine(torch_mod, pkg, eng, blocks, 2048, x, fuse=fuse, layout=layout)
    assert cases.sha256(y) == cases.CONTRACT_GOLDEN_SHA256


def test_gen_vector_cases_through_gemv_dev(torch_mod, pkg, oracle, golden):
    """hls/int4_core/gen_vectors.py's cases through gemv_dev_run, as bench_gemv2.c:47-74 checks them."""
    from llm_kv260_b200 import q4_0 as gpu
    for (k, rows, w, x), rec in zip(cases.gen_vector_inputs(), golden["gen_vectors"]):
        blocks = oracle.quantize_q4_0(w)
        xq, xd = oracle.quantize_q8_0(x)
        y = gpu.gemv_q4_0(blocks, k, xq, xd)
        bad = int(np.count_nonzero(_bits(y) != _bits(_y(rec["y"]))))
        assert bad == 0, f"k={k} rows={rows}: {bad}/{rows} rows differ"


def test_config0_through_reference_named_api(torch_mod, oracle, golden):
    from llm_kv260_b200 import q4_0 as gpu
    rec = golden["config0"]
    blocks = oracle.quantize_q4_0(cases.shape_weights(rec["n"], rec["k"], rec["seed"]))
    y = gpu.gemv_q4_0_f32(blocks, rec["k"], cases.shape_x(rec["k"], rec["seed"]))
    assert np.array_equal(_bits(y), _bits(_y(rec["y"])))


@pytest.mark.parametrize("name,n,k,seed", cases.LLAMA_1B_SHAPES)
def test_llama_1b_shapes(torch_mod, pkg, eng, oracle, golden, name, n, k, seed):
    """BASELINE config 1, unsharded, every shape (lm_head included), both x paths."""
    rec = golden["shapes"][name]
    blocks = oracle.quantize_q4_0(cases.shape_weights(n, k, seed))
    assert cases.sha256(blocks) == rec["sha256_blocks"]
    x = cases.shape_x(k, seed)
    for layout in (0, 1):
        for fuse in (0, 1):
            y = _run_engine(torch_mod, pkg, eng, blocks, k, x, fuse=fuse, layout=layout)
            assert cases.sha256(y) == rec["sha256_y"], (layout, fuse)
        y = _run_engine(torch_mod, pkg, eng, blocks, k, x, packed=True, oracle=oracle, layout=layout)
        assert cases.sha256(y) == rec["sha256_y"], layout


@pytest.mark.parametrize("name", sorted(cases.K_SPLIT))
@pytest.mark.parametrize("parts", cases.SPLITS)
def test_ksplit_shards_with_ordered_sum(torch_mod, pkg, eng, oracle, golden, name, parts):
    """Each rank's column shard on the GPU, summed in rank order (tp_llama.cpp:515-521)."""
    _, n, k, seed = next(s for s in cases.LLAMA_1B_SHAPES if s[0] == name)
    blocks = oracle.quantize_q4_0(cases.shape_weights(n, k, seed))
    x = cases.shape_x(k, seed)
    kk = k // parts
    partials = [_run_engine(torch_mod, pkg, eng, cases.k_slice_blocks(blocks, k, r, parts), kk,
                            np.ascontiguousarray(x[r * kk:(r + 1) * kk]), layout=r % 2) for r in range(parts)]
    assert cases.sha256(oracle.allreduce_ordered(partials)) == golden["shapes"][name][f"sha256_ksplit{parts}"]


# ------------------------------------------------------------ shapes and edges

@pytest.mark.parametrize("k", [256, 512, 768, 1024, 1536, 2048, 2560, 3072, 4096, 6144, 7936, 8192])
@pytest.mark.parametrize("rows", [1, 3, 17, 257])
def test_every_team_width_and_blocks_per_thread(torch_mod, pkg, eng, oracle, k, rows):
    """nb = 8..256 covers teams of 8/16/32 threads and 1..8 blocks per thread; ragged row counts."""
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 1000 + k + rows))
    x = cases.std_weights(1, k, 2000 + k)[0]
    want = oracle.gemv_q4_0_f32(blocks, k, x)
    for layout, fuse, ks in [(0, 0, 1), (0, 1, 1), (1, 0, 1), (1, 1, 1), (1, 0, 2), (1, 1, 4)]:
        got = _run_engine(torch_mod, pkg, eng, blocks, k, x, fuse=fuse, layout=layout, kslices=ks)
        assert np.array_equal(_bits(got), _bits(want)), f"k={k} rows={rows} fuse={fuse} layout={layout} ks={ks}"


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("k", [2048, 8192])
@pytest.mark.parametrize("stage_bytes,stages,ctas,ks", [(16, 1, 1, 1), (1152, 2, 1, 2), (4096, 3, 4, 4),
                                                        (65536, 2, 2, 1), (16384, 8, 2, 2), (200000, 1, 1, 4)])
def test_pipeline_shapes_do_not_change_bits(torch_mod, pkg, eng, oracle, stage_bytes, stages, ctas, ks, k, layout):
    blocks = oracle.quantize_q4_0(cases.std_weights(1000, k, 31))
    x = cases.std_weights(1, k, 32)[0]
    want = oracle.gemv_q4_0_f32(blocks, k, x)
    got = _run_engine(torch_mod, pkg, eng, blocks, k, x, stage_bytes=stage_bytes, stages=stages, ctas_per_sm=ctas,
                      kslices=ks, layout=layout)
    assert np.array_equal(_bits(got), _bits(want))


@pytest.mark.parametrize("k", [2048, 8192])
@pytest.mark.parametrize("stages", [1, 3, 5])
def test_many_groups_per_cta_with_odd_stage_requests(torch_mod, pkg, eng, oracle, stages, k):
    """Tile layout, one CTA per SM and at least 6 row groups per CTA: the ring
    wraps several times for each consumer quad, whatever stage count is asked."""
    rows = 16 * 148 * 6 + 5
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 77 + stages))
    x = cases.std_weights(1, k, 78)[0]
    want = oracle.gemv_q4_0_f32(blocks, k, x)
    for fuse in (0, 1):
        got = _run_engine(torch_mod, pkg, eng, blocks, k, x, fuse=fuse, stages=stages, ctas_per_sm=1, layout=1)
        assert np.array_equal(_bits(got), _bits(want)), (stages, fuse)


def test_zero_and_degenerate_activations(torch_mod, pkg, eng, oracle):
    """All-zero x (d = 0, inv = 0), negative zeros, tiny values, zero weight blocks."""
    k = 512
    w = cases.std_weights(64, k, 41)
    w[5] = 0.0
    w[9, :32] = -0.0
    blocks = oracle.quantize_q4_0(w)
    edge = cases.q8_edge_inputs()
    for x in (np.zeros(k, np.float32), np.full(k, -0.0, np.float32), np.tile(edge["tiny"], k // 32),
              np.tile(edge["floor_half"], k // 32), np.tile(edge["roundf_tie"], k // 32)):
        want = oracle.gemv_q4_0_f32(blocks, k, x)
        for layout in (0, 1):
            for fuse in (0, 1):
                got = _run_engine(torch_mod, pkg, eng, blocks, k, x, fuse=fuse, layout=layout)
                assert np.array_equal(_bits(got), _bits(want))


# ------------------------------------------------------------ quantiser

@pytest.mark.parametrize("name", sorted(cases.q8_edge_inputs()))
def test_q8_quantiser_edges_match_reference(torch_mod, golden, name):
    from llm_kv260_b200 import q4_0 as gpu
    q, d = gpu.quantize_q8_0(cases.q8_edge_inputs()[name])
    assert q.tolist() == golden["q8_edges"][name]["q"]
    assert d.view(np.uint16).tolist() == golden["q8_edges"][name]["d_bits"]


def test_q8_quantiser_random_and_roundf_mode(torch_mod, oracle, golden):
    from llm_kv260_b200 import q4_0 as gpu
    x = cases.std_weights(1, 8192, 1)[0]
    q, d = gpu.quantize_q8_0(x)
    assert cases.sha256(q) == golden["q8_random"]["sha256_q"]
    assert cases.sha256(d) == golden["q8_random"]["sha256_d"]
    half = cases.q8_edge_inputs()["floor_half"]
    qr, _ = gpu.quantize_q8_0(half, round_mode=1)
    qo, _ = oracle.quantize_q8_0(half, oracle.ROUND_ROUNDF)
    assert np.array_equal(qr, qo) and qr[1] == 0


# ------------------------------------------------------------ drop-in interfaces

def test_gemv_dev_start4_staggered_quarters(torch_mod, pkg, oracle):
    """gemv_dev_start4 (gemv_dev.h:35): four quarters at unrelated, staggered addresses."""
    torch = torch_mod
    rows, k = 512, 2048
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 51))
    x = cases.std_weights(1, k, 52)[0]
    xq, xd = oracle.quantize_q8_0(x)
    rb = k // 32 * 18
    q = rows // 4
    bufs = []
    for m in range(4):
        pad = (m & 1) * 16384
        t = torch.zeros(pad + q * rb + 64, dtype=torch.uint8, device="cuda")
        t[pad:pad + q * rb] = torch.from_numpy(blocks[m * q:(m + 1) * q].reshape(-1).copy()).cuda()
        bufs.append((t, int(t.data_ptr()) + pad))
    xp = _dev(torch, oracle.pack_x_for_engine(xq, xd))
    y = torch.full((rows,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    dev = pkg.GemvDev("gemv_q4_0:0")
    dev.start4([a for _, a in bufs], int(xp.data_ptr()), int(y.data_ptr()), k, rows)
    dev.wait()
    dev.close()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(oracle.gemv_q4_0(blocks, k, xq, xd)))


@pytest.mark.parametrize("rows,k", [(32, 256), (64, 512), (768, 2048), (2048, 512), (32, 8192)])
def test_gemv2_fetch_and_mac_over_chunk_pairs(torch_mod, pkg, oracle, rows, k):
    """gemv2 (gemv2_dev.h): port regions in the chunk-pair interleave, fetch then mac."""
    torch = torch_mod
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 61 + rows))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, k, 62)[0])
    rb, nch, q = k // 32 * 18, k // 256, rows // 4
    regions = [np.zeros(q * rb, np.uint8) for _ in range(4)]
    for r in range(rows):
        for c in range(nch):
            off, port = oracle.gemv2_chunk_offset(r, c, rows, k)
            regions[port][off:off + 144] = blocks[r, c * 144:(c + 1) * 144]
    dev_regions = [torch.from_numpy(reg).cuda() for reg in regions]
    xp = _dev(torch, oracle.pack_x_for_engine(xq, xd))
    y = torch.full((rows,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    g2 = pkg.Gemv2Dev()
    g2.fetch_start([int(t.data_ptr()) for t in dev_regions], k, rows)
    g2.mac_start(int(xp.data_ptr()), int(y.data_ptr()), k, rows)
    g2.mac_wait()
    assert g2.mac_idle()
    with pytest.raises(pkg.B200Error):          # a mac with no pending fetch is refused
        g2.mac_start(int(xp.data_ptr()), int(y.data_ptr()), k, rows)
    g2.drain()
    g2.close()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(oracle.gemv_q4_0(blocks, k, xq, xd)))


def test_udmabuf_pool_clean_run_invalidate(torch_mod, pkg, oracle):
    """The reference's call pattern (tp_llama.cpp:355-374): CPU writes the pool,
    clean, run on device addresses, invalidate, CPU reads."""
    rows, k = 256, 1024
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 71))
    xq, xd = oracle.quantize_q8_0(cases.std_weights(1, k, 72)[0])
    xp = oracle.pack_x_for_engine(xq, xd)
    pool = pkg.Udmabuf("udmabuf0", size=8 << 20, device=0)
    w_h = pool.alloc(blocks.nbytes, 64 << 10)
    x_h = pool.alloc(xp.nbytes + 64, 4096)
    y_h = pool.alloc(rows * 4, 4096)
    pool.view(w_h, blocks.nbytes)[:] = blocks.reshape(-1)
    pool.view(x_h, xp.nbytes)[:] = xp
    pool.clean(w_h, blocks.nbytes)
    pool.clean(x_h, xp.nbytes)
    pool.invalidate(y_h, rows * 4)
    dev = pkg.GemvDev()
    dev.run(pool.phys(w_h), pool.phys(x_h), pool.phys(y_h), k, rows)
    pool.invalidate(y_h, rows * 4)
    y = pool.view(y_h, rows * 4).copy().view(np.float32)
    dev.close()
    pool.close()
    assert np.array_equal(_bits(y), _bits(oracle.gemv_q4_0(blocks, k, xq, xd)))


def test_repack_layout_matches_its_definition(torch_mod, pkg, eng, oracle):
    """Tile (g, c) at ((g*nch)+c)*2304: nibbles [row][lane][16], then scales [row][lane]; padded rows zero."""
    torch = torch_mod
    rows, k = 37, 512
    blocks = oracle.quantize_q4_0(cases.std_weights(rows, k, 81))
    T = eng.repack(pkg.QMat(_dev(torch, blocks), rows, k))
    eng.sync()
    tiles = T.blocks.cpu().numpy()
    nb, nch = k // 32, k // 256
    assert tiles.size == pkg.tiled_bytes(rows, k) == 48 * nb * 18
    for r in range(48):
        for b in range(nb):
            g, i, c, l = r // 16, r % 16, b // 8, b % 8
            base = (g * nch + c) * 2304
            nib = tiles[base + (i * 8 + l) * 16: base + (i * 8 + l) * 16 + 16]
            sc = tiles[base + 2048 + (i * 8 + l) * 2: base + 2048 + (i * 8 + l) * 2 + 2]
            if r < rows:
                assert np.array_equal(nib, blocks[r, b * 18 + 2:b * 18 + 18])
                assert np.array_equal(sc, blocks[r, b * 18:b * 18 + 2])
            else:
                assert not nib.any() and not sc.any()


def test_bad_arguments_are_refused(torch_mod, pkg, oracle):
    torch = torch_mod
    e = pkg.Engine(0)
    w = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, dtype=torch.float32, device="cuda")
    y = torch.zeros(16, dtype=torch.float32, device="cuda")
    with pytest.raises(pkg.B200Error, match="-22"):
        e.gemv_f32(pkg.QMat(w, 16, 128), x, y)                  # nb = 4, not a multiple of 8 lanes
    with pytest.raises(pkg.B200Error, match="-22"):
        e.gemv_f32(pkg.QMat(int(w.data_ptr()), 1, 16384), torch.zeros(16384, device="cuda"), y)   # above 8192
    with pytest.raises(pkg.B200Error, match="-22"):
        e.gemv_f32(pkg.QMat(int(w.data_ptr()) + 2, 1, 256), x, y)    # misaligned weights
    e.close()
    dev = pkg.GemvDev()
    with pytest.raises(pkg.B200Error):
        dev.start4([int(w.data_ptr())] * 4, int(x.data_ptr()), int(y.data_ptr()), 256, 6)   # rows % 4
    dev.close()
