"""Kernel-level parity of the CUDA path against the oracle, through the C ABI entry points
(vg_k_*) on raw device pointers."""
import numpy as np
import pytest

from conftest import assert_close
from oracle import oracle as O
from voxgen_b200 import api, gguf, synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
Q8, F16 = gguf.GGML_Q8_0, gguf.GGML_F16


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check(rc):
    assert rc == 0, api.STATUS.get(rc, rc)


def packed_matrix(dtype, raw, rows, cols):
    import ctypes
    b = ctypes.c_uint64()
    check(api.lib().vg_k_packed_bytes(dtype, rows, cols, ctypes.byref(b)))
    packed = torch.zeros(b.value, dtype=torch.uint8, device="cuda")
    src = dev(raw.view(np.uint8))
    check(api.lib().vg_k_repack(dtype, src.data_ptr(), rows, cols, packed.data_ptr(), None))
    return packed


def make_matrix(rng, dtype, rows, cols):
    return synth.q8_matrix(rng, rows, cols) if dtype == Q8 else synth.f16_matrix(rng, rows, cols).view(np.uint8)


@pytest.mark.parametrize("dtype,rows,cols", [
    (Q8, 1, 32), (Q8, 7, 64), (Q8, 5, 96), (Q8, 1000, 1024), (Q8, 1281, 2048), (Q8, 513, 2080),
    (Q8, 2048, 6144), (Q8, 12288, 2048),
    (F16, 5, 8), (F16, 3, 24), (F16, 300, 1024), (F16, 129, 1000), (F16, 2048, 6144),
])
def test_matvec(dtype, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    raw = make_matrix(rng, dtype, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    alpha = 0.75
    want = O.matvec(dtype, raw.view(np.uint8), rows, cols, x, alpha)
    packed = packed_matrix(dtype, raw, rows, cols)
    xd = dev(x)
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    check(api.lib().vg_k_matvec(dtype, packed.data_ptr(), rows, cols, xd.data_ptr(), y.data_ptr(), alpha, None))
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), want, what=f"matvec {dtype} {rows}x{cols}")


@pytest.mark.parametrize("dtype,rows,cols", [(Q8, 2048, 6144), (Q8, 12288, 2048), (Q8, 1281, 2048),
                                              (F16, 2048, 6144), (F16, 300, 1024)])
@pytest.mark.parametrize("zero_column", [False, True])
def test_matvec_outlier(dtype, rows, cols, zero_column):
    """x with one element 1000x the rms of the others. The Q8_0 operand shares one power of two
    over the whole vector, so the outlier sets the digits' resolution for every element. With
    zero_column the outlier's weight column is zero: the products are then all small and the
    quantisation error of the small elements is measured against small outputs."""
    rng = np.random.default_rng(rows * 11 + cols + zero_column)
    raw = make_matrix(rng, dtype, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    k = int(rng.integers(cols))
    x[k] = 1000.0
    if zero_column:
        if dtype == Q8:
            blocks = raw.view(np.uint8).reshape(rows, cols // 32, 34)
            blocks[:, k // 32, 2 + k % 32] = 0
        else:
            raw.view(np.float16).reshape(rows, cols)[:, k] = 0
    want = O.matvec(dtype, raw.view(np.uint8), rows, cols, x, 1.0)
    packed = packed_matrix(dtype, raw, rows, cols)
    xd = dev(x)
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    check(api.lib().vg_k_matvec(dtype, packed.data_ptr(), rows, cols, xd.data_ptr(), y.data_ptr(), 1.0, None))
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), want, what=f"matvec {dtype} {rows}x{cols} outlier (zero column {zero_column})")


def tile_offsets(rows, cols, q8):
    """Byte offsets of the segmented 16-row tile layout (mirror of TileGeom in kernels.cuh): a
    K-step of 16 rows x 32 bytes is four 8x16-byte matrices [rows 0-7 | rows 8-15] x [bytes 0-15 |
    bytes 16-31]; 8 K-steps and then (Q8_0) their scales [row % 8][K-step][row / 8] per segment."""
    step = 32 if q8 else 16
    seg_cols = 8 * step
    nseg = -(-cols // seg_cols)
    seg_bytes = 4096 + (256 if q8 else 0)
    r = np.arange(rows)[:, None]
    k = np.arange(cols)[None, :]
    seg, kk = k // seg_cols, k % seg_cols
    kb = (kk % step) * (1 if q8 else 2)
    tr = r % 16
    base = ((r // 16) * nseg + seg) * seg_bytes
    elem = base + (kk // step) * 512 + ((kb >> 4) * 2 + (tr >> 3)) * 128 + (tr & 7) * 16 + (kb & 15)
    b = np.arange(cols // 32)[None, :]
    scale = ((r // 16) * nseg + b // 8) * seg_bytes + 4096 + (tr & 7) * 32 + (b % 8) * 4 + (tr >> 3) * 2
    return elem, scale, (-(-rows // 16)) * nseg * seg_bytes


@pytest.mark.parametrize("dtype,rows,cols", [(Q8, 6, 64), (Q8, 17, 544), (Q8, 40, 1024), (F16, 9, 272), (F16, 33, 640)])
def test_repack_layout(dtype, rows, cols):
    rng = np.random.default_rng(1)
    raw = make_matrix(rng, dtype, rows, cols)
    packed = packed_matrix(dtype, raw, rows, cols).cpu().numpy()
    elem, scale, total = tile_offsets(rows, cols, dtype == Q8)
    assert packed.size == total
    used = np.zeros(total, bool)
    if dtype == Q8:
        d, qs = gguf.q8_0_unpack(raw, rows, cols)
        assert np.array_equal(packed[elem].view(np.int8), qs)
        lo, hi = packed[scale], packed[scale + 1]
        assert np.array_equal((lo.astype(np.uint16) | (hi.astype(np.uint16) << 8)).view(np.float16), d)
        used[elem] = True
        used[scale] = used[scale + 1] = True
    else:
        h = raw.view(np.uint8).reshape(rows, cols * 2)
        assert np.array_equal(packed[elem], h[:, 0::2]) and np.array_equal(packed[elem + 1], h[:, 1::2])
        used[elem] = used[elem + 1] = True
    assert not packed[~used].any(), "padding bytes must be zero"


@pytest.mark.parametrize("dtype,cols", [(Q8, 1024), (Q8, 2048), (F16, 1024), (F16, 2048)])
def test_embedding_bit_exact(dtype, cols):
    rows = 37
    rng = np.random.default_rng(cols)
    raw = make_matrix(rng, dtype, rows, cols)
    packed = packed_matrix(dtype, raw, rows, cols)
    for tok, alpha in ((0, 1.0), (36, 1.0), (17, 12.0)):
        out = torch.empty(cols, dtype=torch.float32, device="cuda")
        check(api.lib().vg_k_embedding(dtype, packed.data_ptr(), rows, cols, tok, alpha, out.data_ptr(), None))
        torch.cuda.synchronize()
        want = O.embedding(dtype, raw.view(np.uint8), cols, tok, alpha)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    out = torch.empty(cols, dtype=torch.float32, device="cuda")
    assert api.lib().vg_k_embedding(dtype, packed.data_ptr(), rows, cols, rows, 1.0, out.data_ptr(), None) == -5


@pytest.mark.parametrize("n,with_branch", [(1024, False), (2048, True), (96, True), (4096, True)])
def test_residual_rmsnorm(n, with_branch):
    rng = np.random.default_rng(n)
    h = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    w = synth.norm_vector(rng, n)
    hd, bd, wd = dev(h), dev(b), dev(w)
    y = torch.empty(n, dtype=torch.float32, device="cuda")
    check(api.lib().vg_k_residual_rmsnorm(hd.data_ptr(), bd.data_ptr() if with_branch else None, wd.data_ptr(),
                                          n, 1e-5, 0.5, y.data_ptr(), None))
    torch.cuda.synchronize()
    if with_branch:
        hw, yw = O.residual_rmsnorm(h, b, w, 1e-5, 0.5)
        assert_close(hd.cpu().numpy(), hw, atol=1e-6, rtol=1e-6, what="hidden")
    else:
        yw = O.rmsnorm(h, w, 1e-5)
    assert_close(y.cpu().numpy(), yw, what="norm")


@pytest.mark.parametrize("heads,kv_heads,head_dim,ctx,positions", [
    (16, 2, 128, 4352, [0, 1, 15, 16, 17, 271, 272, 1023, 4351]),
    (16, 2, 64, 600, [0, 5, 37, 599]),
    (8, 2, 32, 100, [0, 63, 99]),
    (4, 4, 256, 300, [0, 150, 299]),
    (32, 1, 128, 2100, [2099]),
])
def test_attention(heads, kv_heads, head_dim, ctx, positions):
    rng = np.random.default_rng(heads * ctx + head_dim)
    kvd = kv_heads * head_dim
    k_ref = rng.standard_normal((ctx, kvd)).astype(np.float16)
    v_ref = rng.standard_normal((ctx, kvd)).astype(np.float16)
    # device cache is head-major [kv_head][ctx][head_dim]
    k_hm = np.ascontiguousarray(k_ref.reshape(ctx, kv_heads, head_dim).transpose(1, 0, 2))
    v_hm = np.ascontiguousarray(v_ref.reshape(ctx, kv_heads, head_dim).transpose(1, 0, 2))
    kd, vd = dev(k_hm.view(np.int16)), dev(v_hm.view(np.int16))
    for pos in positions:
        q = (rng.standard_normal(heads * head_dim) * 0.3).astype(np.float32)
        want, _ = O.attention(q, k_ref.view(np.uint16), v_ref.view(np.uint16), heads, kv_heads, head_dim, pos)
        qd = dev(q)
        out = torch.full((heads * head_dim,), float("nan"), dtype=torch.float32, device="cuda")
        check(api.lib().vg_k_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), heads, kv_heads, head_dim,
                                       ctx, pos, out.data_ptr(), None))
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), want, what=f"attention pos={pos}")
