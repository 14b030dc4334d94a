"""The W4A16 matmul on packed weights through the C ABI: the packed weight
layout byte for byte against a numpy restatement, and the matmul against the
oracle restatement of MLX's qmm -- on the register-dequant GEMV kernel
(mma.sync; passes of up to 8 tokens by default, 16 with IAM_QMM_GEMV_MAX_M=16)
and on the tensor-core kernel (tcgen05, weights dequantized into tensor
memory; wider passes, or every pass with IAM_QMM_GEMV_MAX_M=0).

Tolerance as for iam_qmm_affine4: both sides multiply x with the bf16 weights
bf16(q * scale + bias); only the fp32 accumulation order differs, so relative
error <= 1e-2 and cosine >= 0.9999.
"""
import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth

from gpu_util import assert_close_bf16, dev, empty_u16, host_u16, ptr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

u = O.to_u16

ROWS, BLOCK_K, CODE_BYTES, BLOCK_BYTES = 128, 256, 16384, 18432


def swz(r):
    """The chunk swizzle of qmm.cuh (qp_swz): a bijection of r % 8."""
    return ((r & 3) << 1) | ((r >> 2) & 1)


def pack_ref(w, s, b):
    """numpy restatement of the packed layout (qmm.cuh): tiles of 128 rows x
    256 k, codes row-major with 16-byte chunks swizzled by (chunk ^ swz(row)),
    nibble s of a word = k 2s, nibble s+4 = k 2s+1; (scale | bias << 16) words
    after the codes; then one flag byte a tile (padded to 256 bytes): 1 when
    every scale of the tile is below 0.5 in magnitude, and then the tile's
    scales are stored times 2^129."""
    N, KW = w.shape
    K = KW * 8
    KB = -(-K // BLOCK_K)
    T = -(-N // ROWS)
    out = np.zeros((T, KB, BLOCK_BYTES), np.uint8)
    nib = (w[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15  # [N, KW, 8] k order
    perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])  # stored nibble p holds k perm[p]
    words = np.zeros((N, KB * 32), np.uint32)
    words[:, :KW] = (nib[:, :, perm] << (4 * np.arange(8, dtype=np.uint32))).sum(axis=2, dtype=np.uint32)
    G = K // 64
    s16 = s.view(np.uint16)
    flags = np.ones(T, np.uint8)
    for t in range(T):
        if np.any(((s16[t * ROWS:(t + 1) * ROWS] >> 7) & 0xFF) >= 126):
            flags[t] = 0
    # the products (|s| < 0.5) stay below the float32 and bf16 maxima
    with np.errstate(over="ignore"):
        s_big = (s.astype(np.float64) * 2.0 ** 129).astype(np.float32).astype(synth.BF16).view(np.uint16)
    s_st = np.where(np.repeat(flags, ROWS)[:N, None] == 1, s_big, s16)
    sb = np.zeros((N, KB * 4), np.uint32)
    sb[:, :G] = s_st.astype(np.uint32) | (b.view(np.uint16).astype(np.uint32) << 16)
    for r in range(N):
        t, tr = divmod(r, ROWS)
        for kb in range(KB):
            blk = out[t, kb]
            chunks = words[r, kb * 32:(kb + 1) * 32].reshape(8, 4)
            for c in range(8):
                o = tr * 128 + ((c ^ swz(tr)) << 4)
                blk[o:o + 16] = chunks[c].view(np.uint8)
            blk[CODE_BYTES + tr * 16:CODE_BYTES + tr * 16 + 16] = sb[r, kb * 4:kb * 4 + 4].view(np.uint8)
    tail = np.zeros(-(-T // 256) * 256, np.uint8)
    tail[:T] = flags
    return np.concatenate([out.reshape(-1), tail])


def pack_dev(w, s, b, N, K):
    nbytes = I.qmm_packed_bytes(N, K)
    assert nbytes == -(-N // ROWS) * -(-K // BLOCK_K) * BLOCK_BYTES + -(-(-(-N // ROWS)) // 256) * 256
    packed = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    keep = [dev(w, torch), dev(s.view(np.uint16), torch), dev(b.view(np.uint16), torch)]
    I.qmm_pack_affine4(*[ptr(t) for t in keep], ptr(packed), N, K)
    torch.cuda.synchronize()
    return packed


def big_scales(s, rows):
    """Scales of `rows` raised to 0.6 in one group each: those tiles take the
    general conversion (no 2^129 pre-scaling)."""
    s = s.copy()
    s[rows, 1] = synth.BF16(0.6)
    return s


def test_pack_layout_matches_restatement():
    N, K = 200, 640  # a partial tile and a partial k block
    w, s, b = synth.gen_qweight(21, "t.pack", N, K)
    got = pack_dev(w, s, b, N, K).cpu().numpy()
    ref = pack_ref(w, s, b)
    assert ref[-256] == 1  # small scales: the fast conversion
    assert np.array_equal(got, ref)
    s2 = big_scales(s, [150])  # second tile only
    got = pack_dev(w, s2, b, N, K).cpu().numpy()
    ref = pack_ref(w, s2, b)
    assert ref[-256] == 1 and ref[-255] == 0
    assert np.array_equal(got, ref)


@pytest.fixture(params=["default", "tensor_core", "gemv16", "gemv_16warps"])
def kernel(request, monkeypatch):
    """The library's kernel choice (GEMV up to 8 tokens), the tensor-core
    kernel at every width, the GEMV kernel up to 16 tokens (its 16-token
    tile), or the GEMV kernel with 16 consumer warps instead of 8."""
    if request.param == "tensor_core":
        monkeypatch.setenv("IAM_QMM_GEMV_MAX_M", "0")
    elif request.param == "gemv16":
        monkeypatch.setenv("IAM_QMM_GEMV_MAX_M", "16")
    elif request.param == "gemv_16warps":
        monkeypatch.setenv("IAM_QMM_GEMV_MAX_M", "16")
        monkeypatch.setenv("IAM_QMM_GEMV_WARPS", "16")
    return request.param


@pytest.mark.parametrize("M", [1, 8, 16, 32, 64])
def test_qmm_packed_mixed_tiles(M, kernel):
    """Tiles with a scale >= 0.5 use the general conversion, the others the
    2^129 pre-scaled one; both must match the oracle."""
    N, K = 512, 1024
    w, s, b = synth.gen_qweight(61, "t.tc.mixed", N, K)
    s = big_scales(s, [5, 300])  # tiles 0 and 2
    x = synth.gen_normal_bf16(62, f"t.tc.mixed.x.{M}", M * K, 1.0).astype(np.float32).reshape(M, K)
    ref = O.qmm_affine4(x, w, s.astype(np.float32), b.astype(np.float32))
    packed = pack_dev(w, s, b, N, K)
    flags = packed.cpu().numpy()[-256:-252]
    assert list(flags) == [0, 1, 0, 1]
    dx = dev(u(x), torch)
    y = empty_u16(torch, M, N)
    I.qmm_affine4_packed(ptr(packed), ptr(dx), ptr(y), M, N, K)
    torch.cuda.synchronize()
    assert_close_bf16(host_u16(y), ref)


def _case(N, K, M, indep_bias=False, seed=31):
    w, s, b = synth.gen_qweight(seed, f"t.tc.{N}x{K}", N, K)
    if indep_bias:  # biases not tied to the scales
        b = synth.gen_normal_bf16(seed + 1, f"t.tc.b.{N}x{K}", N * K // 64, 0.05).reshape(N, K // 64)
    x = synth.gen_normal_bf16(seed + 2, f"t.tc.x.{M}x{K}", M * K, 1.0).astype(np.float32).reshape(M, K)
    ref = O.qmm_affine4(x, w, s.astype(np.float32), b.astype(np.float32))
    packed = pack_dev(w, s, b, N, K)
    dx = dev(u(x), torch)
    y = empty_u16(torch, M, N)
    I.qmm_affine4_packed(ptr(packed), ptr(dx), ptr(y), M, N, K)
    torch.cuda.synchronize()
    return host_u16(y), ref


@pytest.mark.parametrize("N,K", [(10240, 5120), (6144, 5120), (48, 5120), (5120, 6144), (1024, 5120)])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 16, 17, 32, 40, 64, 100])
def test_qmm_packed_matches_oracle(N, K, M, kernel):
    got, ref = _case(N, K, M)
    assert_close_bf16(got, ref)


@pytest.mark.parametrize("N,K,M", [(5120, 17408, 4), (5120, 17408, 16), (5120, 17408, 32), (264, 704, 5),
                                   (128, 256, 1), (136, 448, 12)])
def test_qmm_packed_odd_shapes(N, K, M, kernel):
    got, ref = _case(N, K, M, indep_bias=True, seed=41)
    assert_close_bf16(got, ref)


@pytest.mark.parametrize("M", [4, 32])
def test_qmm_packed_repeat_is_deterministic(M):
    """Split-K partials meet in a workspace whose counters the last CTA
    re-zeroes, summed in split order: a second call must give the same bits
    (GEMV kernel at 4 tokens, tensor-core kernel at 32)."""
    w, s, b = synth.gen_qweight(51, "t.tc.rep", 1024, 6144)
    x = synth.gen_normal_bf16(52, f"t.tc.rep.x{M}", M * 6144, 1.0).reshape(M, 6144)
    packed = pack_dev(w, s, b, 1024, 6144)
    dx = dev(x.view(np.uint16), torch)
    ys = []
    for _ in range(2):
        y = empty_u16(torch, M, 1024)
        I.qmm_affine4_packed(ptr(packed), ptr(dx), ptr(y), M, 1024, 6144)
        torch.cuda.synchronize()
        ys.append(host_u16(y))
    assert np.array_equal(ys[0], ys[1])


def test_qmm_packed_rejects_bad_shapes():
    assert I.qmm_packed_bytes(16, 100) == 0
    with pytest.raises(I.IamError):
        I.qmm_affine4_packed(0, 0, 0, 1, 16, 64)
    with pytest.raises(I.IamError):
        I.qmm_pack_affine4(0, 0, 0, 0, 16, 96)


def test_mma_sync_qmm_after_tensor_core_split_k():
    """The tensor-core kernel leaves fp32 partials in its split-K workspace;
    the mma.sync kernel's operator-level workspace must stay zero regardless:
    a split-K tensor-core call followed by a split-K iam_qmm_affine4 call."""
    _case(1024, 6144, 32)  # tensor core, K split over CTAs
    N, K, M = 1024, 5120, 8
    w, s, b = synth.gen_qweight(81, "t.tc.then.sync", N, K)
    x = synth.gen_normal_bf16(82, "t.tc.then.sync.x", M * K, 1.0).astype(np.float32).reshape(M, K)
    ref = O.qmm_affine4(x, w, s.astype(np.float32), b.astype(np.float32))
    keep = [dev(w, torch), dev(s.view(np.uint16), torch), dev(b.view(np.uint16), torch), dev(u(x), torch)]
    y = empty_u16(torch, M, N)
    I.qmm_affine4(*[ptr(t) for t in keep], ptr(y), M, N, K)
    torch.cuda.synchronize()
    assert_close_bf16(host_u16(y), ref)
