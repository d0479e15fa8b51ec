"""dn_gguf_split: GGUF Q4_0 / Q8_0 blocks split on the device into the
engine's layout, against the reference loader's CPU split (gguf.dart:206-215
splitQ4_0: the fp16 scale bytes and the 16 nibble bytes of every 18-byte
block; gguf.dart:269-283 splitQ8_0: the fp16 scale widened to f32, exactly,
and the 32 int8 of every 34-byte block), restated here with numpy. Bit for
bit, including subnormal and infinite scales, on a block count that fills no
launch evenly and on blocks that are 2- but not 4-byte aligned.

dn_gguf_linear_qa: the one-token product straight on the file's blocks, no
split, against lab_gemm (mode 1) on the blocks split as the loader splits
them, bit for bit, up to the whole 151936-row lm_head."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def gguf_blocks(rng, fmt, count):
    size = 18 if fmt == "q4" else 34
    raw = rng.integers(0, 256, count * size, dtype=np.uint8).reshape(count, size)
    scales = rng.uniform(1e-4, 4e-2, count).astype(np.float16)
    special = np.array([0.0, 6e-8, 6.1e-5, -3e-2, 65504.0, np.inf, -np.inf], np.float16)
    scales[: min(count, special.size)] = special[: min(count, special.size)]
    raw[:, :2] = scales.view(np.uint8).reshape(count, 2)
    return raw


def split_like_reference(fmt, raw):
    if fmt == "q4":
        return raw[:, 2:].ravel().copy(), raw[:, :2].ravel().copy()
    return raw[:, 2:].ravel().copy(), raw[:, :2].copy().view(np.float16).astype(np.float32).ravel()


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("count,offset", [(1, 0), (4097, 0), (77777, 2)])
def test_split_matches_the_reference_loader(cuda_lib, fmt, count, offset):
    L = cuda_lib
    rng = np.random.default_rng(count + offset + (fmt == "q4"))
    raw = gguf_blocks(rng, fmt, count)
    # The blocks at a 2-byte (not 4-byte) aligned address when offset is 2.
    src = torch.zeros(raw.size + 16, dtype=torch.uint8, device="cuda")
    src[offset:offset + raw.size] = torch.from_numpy(raw.ravel()).cuda()
    vbytes = 16 if fmt == "q4" else 32
    qs = torch.full((count * vbytes,), 0xAB, dtype=torch.uint8, device="cuda")
    sc = torch.full((count * (2 if fmt == "q4" else 4),), 0xCD, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.dn_gguf_split(1 if fmt == "q4" else 0, src.data_ptr() + offset, count, qs.data_ptr(),
                         sc.data_ptr(), st)
    torch.cuda.synchronize()
    assert rc == 0 and L.dn_device_status(1) == 0
    want_qs, want_sc = split_like_reference(fmt, raw)
    assert np.array_equal(qs.cpu().numpy(), want_qs)
    got_sc = sc.cpu().numpy()
    assert np.array_equal(got_sc, want_sc.view(np.uint8).ravel())


def test_split_rejects_bad_arguments(cuda_lib):
    L = cuda_lib
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    assert L.dn_gguf_split(2, p, 1, p + 64, p + 256, st) == -1         # no such format
    assert L.dn_gguf_split(0, p + 1, 1, p + 64, p + 256, st) == -1     # blocks not 2-byte aligned
    assert L.dn_gguf_split(0, p, 1, p + 66, p + 256, st) == -1         # values not 4-byte aligned
    assert L.dn_gguf_split(0, p, 1, p + 64, p + 258, st) == -1         # Q8 scales not 4-byte aligned
    assert L.dn_gguf_split(0, p, -1, p + 64, p + 256, st) == -1
    assert L.dn_gguf_split(0, 0, 0, 0, 0, st) == 0                      # nothing to do


def gguf_matrix(rng, fmt, rows, cols):
    """A matrix as a GGUF file stores it: rows x cols / 32 blocks, finite fp16
    scales (subnormal, zero and negative ones included); Q8_0 values in
    [-127, 127], as llama.cpp's and dianoia's quantizers write them."""
    raw = gguf_blocks(rng, fmt, rows * (cols // 32))
    sc = raw[:, :2].copy().view(np.float16)
    sc[~np.isfinite(sc)] = np.float16(0.01)
    raw[:, :2] = sc.view(np.uint8)
    if fmt == "q8":
        vals = raw[:, 2:]
        vals[vals == 0x80] = 0x81
    return raw


@pytest.mark.parametrize("fmt,rows,cols", [("q8", 33, 256), ("q8", 1000, 2048), ("q8", 2048, 6144),
                                           ("q4", 4097, 512), ("q4", 6144, 2048), ("q8", 151936, 2048)])
def test_gguf_linear_matches_the_split_product(cuda_lib, oracle, fmt, rows, cols):
    """dn_gguf_linear_qa on the file's blocks equals lab_gemm (mode 1, n = 1)
    on the blocks split as dianoia's loader splits them, bit for bit."""
    from oracle import oracle as orc
    L = cuda_lib
    rng = np.random.default_rng(rows + cols + (fmt == "q4"))
    raw = gguf_matrix(rng, fmt, rows, cols)
    qs, sc = split_like_reference(fmt, raw)
    if fmt == "q4":
        sc = sc.view(np.uint16)
    x = orc.activations(rng, 1, cols)
    want, _, _ = oracle.gemm(fmt, qs, sc, x, rows, cols, 1, 1)
    st = torch.cuda.current_stream().cuda_stream
    blocks = torch.from_numpy(raw.ravel()).cuda()
    xd = torch.from_numpy(x).cuda()
    xa = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(xd.data_ptr(), xa.data_ptr(), 1, cols, cols // 32 * 36, st) == 0
    ys = torch.full((rows + 1,), float("nan"), device="cuda")
    for _ in range(2):
        rc = L.dn_gguf_linear_qa(1 if fmt == "q4" else 0, blocks.data_ptr(), xa.data_ptr(), ys.data_ptr(),
                                 rows, cols, 1, st)
        torch.cuda.synchronize()
        assert rc == 0 and L.dn_device_status(1) == 0
        got = ys.cpu().numpy()
        assert np.array_equal(got[:rows].view(np.uint32), want.view(np.uint32))
        assert np.isnan(got[rows])  # nothing written past the rows


def test_gguf_linear_rejects_bad_arguments(cuda_lib):
    L = cuda_lib
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    assert L.dn_gguf_linear_qa(2, p, p + 4096, p + 8192, 4, 256, 0, st) == -1      # no such format
    assert L.dn_gguf_linear_qa(0, p + 2, p + 4096, p + 8192, 4, 256, 0, st) == -1  # blocks not 16-aligned
    assert L.dn_gguf_linear_qa(0, p, p + 4098, p + 8192, 4, 256, 0, st) == -1      # QA input not 4-aligned
    assert L.dn_gguf_linear_qa(0, p, p + 4096, p + 8192, 4, 224, 0, st) == -1      # Q8_0 cols % 256
    assert L.dn_gguf_linear_qa(1, p, p + 4096, p + 8192, 4, 256, 0, st) == -1      # Q4_0 cols % 512
    assert L.dn_gguf_linear_qa(0, p, p + 4096, p + 8192, 0, 256, 0, st) == 0       # no rows
