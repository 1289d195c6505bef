"""Device kernels against the oracle, through the C ABI.

* dequantization: bit-exact with the reference decoders for every block type;
* the streamed GEMV: within a summation-order tolerance of the reference's
  FMA chain, for every block type, 1..8 positions (and chunked above 8),
  shapes that do and do not fill a tile.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

BLK = {O.Q8_0: (32, 34), O.Q6_K: (256, 210), O.Q5_K: (256, 176), O.Q2_K: (256, 84), O.F32: (1, 4)}
GOLD = {O.Q8_0: "q8_0", O.Q6_K: "q6_k", O.Q5_K: "q5_k", O.Q2_K: "q2_k"}


def random_matrix(dtype, rows, cols, seed, gaussian=True):
    """GGML blocks for a rows x cols matrix: encoded N(0, 0.02) values via a
    synthetic model when gaussian, else raw random blocks with finite scales."""
    rng = np.random.default_rng(seed)
    bv, bb = BLK[dtype]
    nblk = rows * cols // bv
    if dtype == O.F32:
        return rng.normal(0, 0.02, rows * cols).astype(np.float32).view(np.uint8)
    raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    pos = {O.Q8_0: [0], O.Q6_K: [208], O.Q5_K: [0, 2], O.Q2_K: [80, 82]}[dtype]
    for p in pos:
        exp = rng.integers(5, 15, size=nblk).astype(np.uint16)
        h = (rng.integers(0, 2, size=nblk).astype(np.uint16) << 15) | (exp << 10) | rng.integers(0, 1024, size=nblk).astype(np.uint16)
        raw[:, p:p + 2] = h.view(np.uint8).reshape(nblk, 2)
    return raw.reshape(-1)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q6_K, O.Q5_K, O.Q2_K, O.F32])
@pytest.mark.parametrize("rows", [1, 6, 37])
def test_device_dequant_is_bit_exact(cuda, dtype, rows):
    cols = 512 if dtype != O.Q8_0 else 576
    blocks = random_matrix(dtype, rows, cols, seed=rows * 31 + dtype)
    w = eb.Weights(dtype, rows, cols, blocks)
    got = w.dequant(0, rows)
    want = O.decode(dtype, blocks.tobytes()).reshape(rows, cols)
    assert np.array_equal(bits(got), bits(want))
    part = w.dequant(rows // 2, rows - rows // 2)
    assert np.array_equal(bits(part), bits(want[rows // 2:]))


@pytest.mark.parametrize("name", sorted(GOLD.values()))
def test_device_dequant_matches_gguf_py_fixture(cuda, golden, name):
    dtype = {v: k for k, v in GOLD.items()}[name]
    raw = golden[name]
    bv, bb = BLK[dtype]
    nblk = raw.size // bb
    cols = bv * 8 if dtype != O.Q8_0 else 32 * 16
    rows = nblk * bv // cols
    w = eb.Weights(dtype, rows, cols, raw)
    assert np.array_equal(bits(w.dequant(0, rows).reshape(-1)), bits(golden[name + "_out"]))


def gemv_case(cuda, dtype, rows, cols, positions, seed, gaussian=True):
    import torch

    blocks = random_matrix(dtype, rows, cols, seed, gaussian)
    rng = np.random.default_rng(seed + 1)
    x = rng.normal(0, 1, (positions, cols)).astype(np.float32)
    want = O.gemv_fma(dtype, blocks, rows, cols, x, positions)
    w = eb.Weights(dtype, rows, cols, blocks)
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.full((positions, rows), float("nan"), device=cuda)
    w.gemv(xd, positions, yd)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    dense = O.decode(dtype, blocks.tobytes()).reshape(rows, cols)
    scale = np.abs(x) @ np.abs(dense).T  # sum |w x| per output
    return got, want, scale


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q6_K, O.Q5_K, O.Q2_K, O.F32])
@pytest.mark.parametrize("positions", [1, 2, 3, 4, 5, 8])
def test_gemv_matches_the_fma_chain(cuda, dtype, positions):
    rows, cols = (203, 1536) if dtype != O.Q8_0 else (203, 576)
    got, want, scale = gemv_case(cuda, dtype, rows, cols, positions, seed=positions * 7 + dtype)
    err = np.abs(got - want)
    # fp32 summation-order tolerance: relative to sum |w_c x_c| of each output
    assert np.all(err <= 1e-5 * scale + 1e-30), float((err / (scale + 1e-30)).max())


@pytest.mark.parametrize("dtype", [O.Q6_K, O.Q8_0])
def test_gemv_long_rows_split_across_warps(cuda, dtype):
    # few tiles, long rows: the K dimension is split over warps and re-summed
    got, want, scale = gemv_case(cuda, dtype, 8, 12288, 2, seed=99)
    assert np.all(np.abs(got - want) <= 1e-5 * scale)


def test_gemv_more_than_eight_positions_is_chunked(cuda):
    got, want, scale = gemv_case(cuda, O.Q6_K, 64, 1024, 11, seed=5)
    assert np.all(np.abs(got - want) <= 1e-5 * scale)


def test_streamed_refuses_short_activations(cuda):
    import torch

    r = configs.TINY["qwen3-q6_k"]
    m = eb.Model(eb.synth_gguf(r), r.shape)
    idx = m.stream_index("blk.0.attn_q.weight")
    info = m.stream_info(idx)
    x = torch.zeros(info["cols"] - 1, device=cuda)
    y = torch.zeros(info["rows"], device=cuda)
    with pytest.raises(eb.SpmError) as e:
        eb.streamed(m, idx, x, 1, y)
    assert e.value.name == "SPM_E_ACTIVATION_LEN"


def test_streamed_one_stream_of_a_model(cuda):
    import torch

    r = configs.TINY["qwen3-q5_k"]
    img = eb.synth_gguf(r)
    m = eb.Model(img, r.shape)
    idx = m.stream_index("blk.1.ffn_down.weight")
    info = m.stream_info(idx)
    t = eb.gguf_find(img, "blk.1.ffn_down.weight")
    blocks = img[t["offset"]: t["offset"] + t["nbytes"]]
    x = np.random.default_rng(3).normal(0, 1, (3, info["cols"])).astype(np.float32)
    want = O.gemv_fma(info["dtype"], blocks, info["rows"], info["cols"], x, 3)
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.zeros(3, info["rows"], device=cuda)
    eb.streamed(m, idx, xd, 3, yd)
    torch.cuda.synchronize()
    dense = O.decode(info["dtype"], blocks.tobytes()).reshape(info["rows"], info["cols"])
    scale = np.abs(x) @ np.abs(dense).T
    assert np.all(np.abs(yd.cpu().numpy() - want) <= 1e-5 * scale)
    # the model's dequant of that stream is the reference decode, bit for bit
    assert np.array_equal(bits(m.dequant_rows(idx, 0, info["rows"])), bits(dense))


@pytest.mark.parametrize("rows,cols,positions", [(8192, 4096, 4), (2048, 12288, 1), (4096, 4096, 3)])
def test_gemv_reuses_ring_slots(cuda, rows, cols, positions):
    # enough tiles per CTA that every shared-memory ring slot is refilled
    # several times (slot counts of 2, 4 and 8 with 2 or 4 consuming warps)
    got, want, scale = gemv_case(cuda, O.Q6_K, rows, cols, positions, seed=rows + cols)
    assert np.all(np.abs(got - want) <= 1e-5 * scale)


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q6_K, O.Q5_K, O.Q2_K, O.F32])
@pytest.mark.parametrize("positions", [16, 37, 130])
def test_many_positions_on_tensor_cores_match_the_fma_chain(cuda, dtype, positions):
    # 16 or more positions run as one tcgen05 product (exact weights, three-part
    # bf16 splits, fp32 accumulation): the same summation-order bar as the GEMV
    rows, cols = (203, 1536) if dtype != O.Q8_0 else (203, 576)
    got, want, scale = gemv_case(cuda, dtype, rows, cols, positions, seed=positions * 3 + dtype)
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * scale + 1e-30), float((err / (scale + 1e-30)).max())


def test_tensor_core_product_large_shape(cuda):
    # several 128-row and 128-position tiles, k split over many stages
    got, want, scale = gemv_case(cuda, O.Q5_K, 600, 4096, 300, seed=123)
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * scale + 1e-30), float((err / (scale + 1e-30)).max())


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q6_K, O.Q5_K, O.Q2_K])
@pytest.mark.parametrize("positions", [1, 5, 8])
def test_gemv_staging_worst_case(cuda, dtype, positions):
    """Activations are staged per 32-value unit as 22-bit block fixed point
    (a power-of-two scale below the unit's largest |x|, three int8 digit
    planes).  Worst case for that staging: in every unit one value of order
    100 and 31 of order 1e-4, so the small ones keep only a few significant
    bits.  Each output must stay within the staging bound -- at most 2^-22 of
    its unit's largest |x| per value (half a step of 2^(e-22) with
    2^(e-1) <= max|x| < 2^e), times |w|, checked at 2^-21 -- on top of
    the fp32 summation-order tolerance, and within 1e-3 of the largest output
    (the logit bar).  One position runs the dp4a loop; five and eight the
    tensor-core loops (Q8_0: codes as B; K-quants: codes as A)."""
    import torch

    rows, cols = (203, 1536) if dtype != O.Q8_0 else (203, 576)
    rng = np.random.default_rng(1000 + dtype * 10 + positions)
    blocks = random_matrix(dtype, rows, cols, seed=dtype * 17 + positions)
    x = rng.normal(0, 1e-4, (positions, cols)).astype(np.float32)
    units = cols // 32
    big = rng.integers(0, 32, size=(positions, units)) + 32 * np.arange(units)
    for p in range(positions):
        x[p, big[p]] = rng.normal(0, 100, units).astype(np.float32)
    want = O.gemv_fma(dtype, blocks, rows, cols, x, positions)
    w = eb.Weights(dtype, rows, cols, blocks)
    yd = torch.full((positions, rows), float("nan"), device=cuda)
    w.gemv(torch.from_numpy(x).to(cuda), positions, yd)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    dense = np.abs(O.decode(dtype, blocks.tobytes()).reshape(rows, cols))
    scale = np.abs(x) @ dense.T
    umax = np.repeat(np.abs(x).reshape(positions, units, 32).max(axis=2), 32, axis=1)  # unit max per column
    staging = umax @ dense.T * 2.0 ** -21
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * scale + staging + 1e-30), float((err / (1e-5 * scale + staging + 1e-30)).max())
    assert np.all(err <= 1e-3 * np.abs(want).max(axis=1, keepdims=True))
