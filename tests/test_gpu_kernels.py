"""Kernel-level parity on the B200: the tcgen05 TF32 GEMM (all epilogues) and
the attention kernel, each against an exact reference on the same inputs.

TF32 tolerance: a tensor-core product rounds each operand to 10 explicit
mantissa bits, so |C - C_exact| <= 2^-9 * (|A| |B|^T) + FP32 accumulation
slack; the tests assert 3 * 2^-10 * (|A| |B|^T) + 1e-6 elementwise.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TF32_BOUND = 3.0 * 2.0 ** -10
# FP16-operand GEMMs (flag bit 2): the operands the tensor core multiplies are
# exactly _f16_rows(A), _f16_rows(B); only FP32 accumulation error remains
ACC_BOUND = 2.0 ** -18


def _f16_rows(X):
    """The device's FP16 operand rows: each row scaled by 2^-e so its largest
    magnitude lies in [2^14, 2^15), rounded to nearest even, scaled back."""
    X = np.ascontiguousarray(X, np.float32)
    mx = np.abs(X).max(axis=1)
    E = np.maximum((mx.view(np.uint32) >> 23) & 0xFF, 1).astype(np.int64)
    e = np.where(mx > 0, np.clip(E - 141, -100, 100), 0)
    s = np.ldexp(1.0, -e)[:, None]
    return (X * s).astype(np.float16).astype(np.float64) / s


def _operands(A, B, flags):
    """(A, B) as the tensor core sees them for exact references, or None."""
    return (_f16_rows(A), _f16_rows(B)) if flags & 4 else None


@pytest.fixture(scope="module")
def lib():
    from svl._abi import load_library

    L = load_library()
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.svl_test_gemm_tf32.argtypes = [P, I, P, I, P, I, I, I, I, I, F, P, I, I, I, I, P]
    L.svl_test_gemm_tf32.restype = I
    L.svl_test_attention.argtypes = [P, I, I, I, I, I, P, P, I, I, I, P, I, P]
    L.svl_test_attention.restype = I
    L.svl_test_gemm_grouped.argtypes = [P, I, P, I, P, I, I, I, I, F, P, P, I, I, P]
    L.svl_test_gemm_grouped.restype = I
    return L


def _gemm(lib, A, B, epi=0, alpha=1.0, aux=None, n_out=0, tf32_tma=0, round_out=0):
    M, K = A.shape
    N = B.shape[0]
    out_cols = n_out if epi == 1 else N
    a = torch.from_numpy(A).cuda()
    b = torch.from_numpy(B).cuda()
    c = torch.full((M, out_cols), float("nan"), device="cuda")
    x = torch.from_numpy(aux).cuda() if aux is not None else None
    rc = lib.svl_test_gemm_tf32(a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), out_cols, M, N, K, epi, alpha,
                                x.data_ptr() if x is not None else None, aux.shape[1] if aux is not None else 0,
                                round_out, n_out, tf32_tma, None)
    assert rc == 0
    return c.cpu().numpy()


SHAPES = [(5, 8, 16), (130, 64, 32), (300, 2048, 512), (257, 512, 2048), (1000, 3072, 512), (129, 768, 512),
          (64, 12288, 512), (4097, 512, 512)]


@pytest.mark.parametrize("M,N,single", [(300, 12288, 0), (129, 3072, 1), (4097, 512, 0), (257, 256, 0),
                                         (64, 12288, 0)])
def test_gemm_grouped_fp16_store(lib, M, N, single):
    """The grouped FP16 store (the PLE projection's per-layer table, the
    full-attention layers' q/k/v): on the same FP16 operands as the FP32 store,
    every stored value is the FP32 result times its (row, 128-column group)
    power of two, rounded to nearest FP16 -- bit for bit; the scale puts the
    group's largest magnitude in [2^14, 2^15] after rounding; the group's sum of squares
    matches the FP32 results'."""
    K = 512
    rng = np.random.default_rng(M + N)
    A = (rng.standard_normal((M, K)) * 10.0 ** rng.uniform(-3, 3, (M, 1))).astype(np.float32)
    B = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    B[: N // 3, :] *= 1e-3  # groups of very different magnitude
    alpha = 0.375
    ref = _gemm(lib, A, B, alpha=alpha, tf32_tma=4 | (2 if single else 0))
    G = N // 128
    a = torch.from_numpy(A).cuda()
    b = torch.from_numpy(B).cuda()
    c16 = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    gi = torch.full((M, G), float("nan"), device="cuda")
    ss = torch.full((M, G), float("nan"), device="cuda")
    rc = lib.svl_test_gemm_grouped(a.data_ptr(), K, b.data_ptr(), K, c16.data_ptr(), N, M, N, K, alpha,
                                   gi.data_ptr(), ss.data_ptr(), G, single, None)
    assert rc == 0
    c16, gi, ss = c16.cpu().numpy(), gi.cpu().numpy(), ss.cpu().numpy()
    assert np.isfinite(gi).all() and np.isfinite(ss).all()
    mant, _ = np.frexp(gi)
    assert (mant == 0.5).all(), "inverse scales must be powers of two"
    scale = (1.0 / gi).astype(np.float32)  # exact: powers of two
    want = (ref.reshape(M, G, 128) * scale[:, :, None]).astype(np.float16).reshape(M, N)
    assert np.array_equal(c16.view(np.uint16), want.view(np.uint16))
    gmax = np.abs(c16.astype(np.float32)).reshape(M, G, 128).max(axis=2)
    nz = gmax > 0
    # the scaled maximum lies in [2^14, 2^15) before the FP16 rounding, which
    # may carry it up to 2^15 itself
    assert (gmax[nz] >= 2.0 ** 14).all() and (gmax[nz] <= 2.0 ** 15).all()
    want_ss = (ref.astype(np.float64).reshape(M, G, 128) ** 2).sum(axis=2)
    assert np.allclose(ss, want_ss, rtol=1e-5, atol=0)  # a 128-term FP32 FMA chain against the f64 sum


@pytest.mark.parametrize("M,N,K", SHAPES)
# bit 0: TFLOAT32 TMA copies, bit 1: one-CTA kernel only, bit 2: FP16 operands with row scales
@pytest.mark.parametrize("tf32_tma", [0, 1, 2, 4, 6])
def test_gemm_store_matches_fp64(lib, M, N, K, tf32_tma):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((N, K), dtype=np.float32)
    if tf32_tma & 4:
        A *= np.exp2(rng.integers(-20, 20, size=(M, 1))).astype(np.float32)  # rows far apart in scale
    C = _gemm(lib, A, B, alpha=0.5, tf32_tma=tf32_tma)
    ref = 0.5 * (A.astype(np.float64) @ B.astype(np.float64).T)
    mag = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64).T
    err = np.abs(C - ref)
    assert np.isfinite(C).all()
    bound = 0.5 * TF32_BOUND * mag + 1e-6 * (1 if not tf32_tma & 4 else mag.max(axis=1, keepdims=True))
    assert (err <= bound).all(), f"max err {err.max()} (bound {bound[err > bound][:3]})"
    ops = _operands(A, B, tf32_tma)
    if ops is not None:
        exact = 0.5 * (ops[0] @ ops[1].T)
        assert (np.abs(C - exact) <= ACC_BOUND * 0.5 * (np.abs(ops[0]) @ np.abs(ops[1]).T) + 1e-30).all()


def test_gemm_operand_rounding_report(lib, capsys):
    """Mean signed error of FLOAT32 vs TFLOAT32 TMA copies (truncation shows as bias)."""
    rng = np.random.default_rng(0)
    A = np.abs(rng.standard_normal((512, 512), dtype=np.float32)) + 1.0
    B = np.abs(rng.standard_normal((512, 512), dtype=np.float32)) + 1.0
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    for mode in (0, 1):
        C = _gemm(lib, A, B, tf32_tma=mode)
        rel = (C - ref) / ref
        print(f"tf32_tma={mode}: mean rel err {rel.mean():.3e}, rms {np.sqrt((rel ** 2).mean()):.3e}")
        assert abs(rel.mean()) < 2e-3


def _interleave_gate_up(gate, up):
    F, K = gate.shape
    F_pad = (F + 127) // 128 * 128
    W = np.zeros((2 * F_pad, K), np.float32)
    for b in range(F_pad // 128):
        rows = slice(b * 128, min(F, (b + 1) * 128))
        n = rows.stop - rows.start
        if n <= 0:
            continue
        W[b * 256: b * 256 + n] = gate[rows]
        W[b * 256 + 128: b * 256 + 128 + n] = up[rows]
    return W


def _gelu64(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978846 * (x + 0.044715 * x ** 3)))


@pytest.mark.parametrize("M,F,K", [(7, 32, 16), (300, 2048, 512), (129, 200, 64), (1000, 200, 64)])
@pytest.mark.parametrize("flags", [0, 2, 4, 6])
def test_gemm_geglu_epilogue(lib, M, F, K, flags):
    rng = np.random.default_rng(F)
    A = rng.standard_normal((M, K), dtype=np.float32) * 0.1
    G = rng.standard_normal((F, K), dtype=np.float32)
    U = rng.standard_normal((F, K), dtype=np.float32)
    W = _interleave_gate_up(G, U)
    out = _gemm(lib, A, W, epi=1, n_out=F, tf32_tma=flags)
    g = A.astype(np.float64) @ G.astype(np.float64).T
    u = A.astype(np.float64) @ U.astype(np.float64).T
    ref = _gelu64(g) * u
    scale = (np.abs(A) @ np.abs(G).T) * (np.abs(A) @ np.abs(U).T)
    assert np.isfinite(out).all()
    assert (np.abs(out - ref) <= 4 * TF32_BOUND * scale + 1e-5).all()


@pytest.mark.parametrize("flags", [0, 4])
def test_gemm_ple_gate_epilogue(lib, flags):
    rng = np.random.default_rng(5)
    M, N, K = 300, 512, 512
    A = rng.standard_normal((M, K), dtype=np.float32) * 0.05
    B = rng.standard_normal((N, K), dtype=np.float32)
    aux = rng.standard_normal((M, 3 * N), dtype=np.float32)
    # the kernel reads aux[row, col]; pass a view starting at column block 1
    aux_view = np.ascontiguousarray(aux)
    a = torch.from_numpy(A).cuda()
    b = torch.from_numpy(B).cuda()
    x = torch.from_numpy(aux_view).cuda()
    c = torch.empty((M, N), device="cuda")
    rc = lib.svl_test_gemm_tf32(a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K, 2, 1.0,
                                x.data_ptr() + N * 4, 3 * N, 0, 0, flags, None)
    assert rc == 0
    acc = A.astype(np.float64) @ B.astype(np.float64).T
    ref = _gelu64(acc) * aux[:, N:2 * N]
    bound = 2 * TF32_BOUND * (np.abs(A) @ np.abs(B).T) * np.abs(aux[:, N:2 * N]) + 1e-6
    assert (np.abs(c.cpu().numpy() - ref) <= bound).all()


def _attention(lib, qkv, lens, nh, kvh, hd, window, impl):
    T = sum(lens)
    ld = qkv.shape[1]
    cu = np.zeros(len(lens) + 1, np.uint64)
    cu[1:] = np.cumsum(lens)
    d_qkv = torch.from_numpy(qkv).cuda()
    d_cu = torch.from_numpy(cu.astype(np.int64)).cuda()
    out = torch.full((T, nh * hd), float("nan"), device="cuda")
    rc = lib.svl_test_attention(d_qkv.data_ptr(), ld, T, nh, kvh, hd, d_cu.data_ptr(), cu.ctypes.data, len(lens),
                                -1 if window is None else window, impl, out.data_ptr(), nh * hd, None)
    assert rc == 0
    return out.cpu().numpy(), cu


def _attention_ref(qkv, lens, cu, nh, kvh, hd, window):
    import oracle

    refs = []
    for b, L in enumerate(lens):
        s, e = int(cu[b]), int(cu[b + 1])
        q = qkv[s:e, : nh * hd]
        k = qkv[s:e, nh * hd: (nh + kvh) * hd]
        v = qkv[s:e, (nh + kvh) * hd:]
        refs.append(oracle.attention(q, k, v, L, nh, kvh, hd, window=window).reshape(L, nh * hd))
    return np.concatenate(refs)


@pytest.mark.parametrize("hd,nh,kvh", [(8, 2, 1), (16, 2, 1), (256, 4, 2), (512, 4, 1)])
@pytest.mark.parametrize("window", [None, 0, 3, 512])
def test_simt_attention_matches_oracle(lib, hd, nh, kvh, window):
    rng = np.random.default_rng(hd + nh)
    lens = [1, 5, 37] if hd > 64 else [1, 5, 37, 70]
    qkv = rng.standard_normal((sum(lens), (nh + 2 * kvh) * hd), dtype=np.float32) * 0.3
    got, cu = _attention(lib, qkv, lens, nh, kvh, hd, window, 0)
    np.testing.assert_allclose(got, _attention_ref(qkv, lens, cu, nh, kvh, hd, window), rtol=2e-5, atol=2e-6)


# impl 1 picks the CTA-pair kernel for head dims 64..256 (multiples of 64)
# with an even query-head group; impl 2 forces the one-CTA kernel.
@pytest.mark.parametrize("hd,nh,kvh", [(32, 2, 1), (64, 2, 1), (128, 4, 2), (256, 4, 2), (256, 8, 2), (256, 2, 2),
                                       (512, 4, 1)])
@pytest.mark.parametrize("window", [None, 0, 5, 100])
@pytest.mark.parametrize("scale", [0.05, 0.6])
@pytest.mark.parametrize("impl", [1, 2])
def test_tensor_core_attention_matches_oracle(lib, hd, nh, kvh, window, scale, impl):
    """TF32 operands: q, k, v, P each carry 2^-11 relative rounding; the
    output tolerance is 4e-3 relative to the largest |v| entry."""
    rng = np.random.default_rng(hd * 7 + nh + int(scale * 10))
    lens = [1, 7, 130, 300]
    qkv = rng.standard_normal((sum(lens), (nh + 2 * kvh) * hd), dtype=np.float32) * scale
    got, cu = _attention(lib, qkv, lens, nh, kvh, hd, window, impl)
    ref = _attention_ref(qkv, lens, cu, nh, kvh, hd, window)
    assert np.isfinite(got).all()
    vmax = np.abs(qkv[:, (nh + kvh) * hd:]).max()
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-3 * vmax)


@pytest.mark.parametrize("impl", [1, 2, 3])
def test_tensor_core_attention_long_sequence_window(lib, impl):
    """2048 tokens with the 512 radius: most key blocks are skipped per query block."""
    rng = np.random.default_rng(21)
    nh, kvh, hd = 4, 2, 256
    lens = [2048, 600]
    qkv = rng.standard_normal((sum(lens), (nh + 2 * kvh) * hd), dtype=np.float32) * 0.1
    got, cu = _attention(lib, qkv, lens, nh, kvh, hd, 512, impl)
    ref = _attention_ref(qkv, lens, cu, nh, kvh, hd, 512)
    vmax = np.abs(qkv[:, (nh + kvh) * hd:]).max()
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-3 * vmax)


def _round_tf32(x):
    """Round-to-nearest, ties away, to 10 explicit mantissa bits (the grid the
    tensor core reads), kept as float32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


@pytest.mark.parametrize("impl", [1, 2, 3])
def test_tensor_core_attention_rescale_and_bounded_rows(lib, impl):
    """Every key block raises each row's score maximum by ~12.8 nats (keys
    carry a shared direction u with weight position / 10, queries carry u),
    so O is rescaled block after block; padding rows of the last query block
    must leave the next sequence's rows untouched.  Inputs sit on the FP16
    grid (hence also on the TF32 grid), so scores are exact and the tolerance
    only covers P's rounding."""
    rng = np.random.default_rng(5)
    nh, kvh, hd = 4, 2, 256
    lens = [70, 511, 129, 385]
    T = sum(lens)
    qkv = rng.standard_normal((T, (nh + 2 * kvh) * hd), dtype=np.float32) * 0.02
    u = rng.standard_normal(hd).astype(np.float32)
    u /= np.linalg.norm(u)
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.float32)
    for h in range(nh):
        qkv[:, h * hd:(h + 1) * hd] += u
    for g in range(kvh):
        c = (nh + g) * hd
        qkv[:, c:c + hd] += (pos / 10.0)[:, None] * u
    qkv[:, (nh + kvh) * hd:] *= 50.0  # values of order 1
    # the FP16 grid (11-bit significand, |x| < 65504) is also on the TF32 grid
    qkv = qkv.astype(np.float16).astype(np.float32)
    got, cu = _attention(lib, qkv, lens, nh, kvh, hd, None, impl)
    ref = _attention_ref(qkv, lens, cu, nh, kvh, hd, None)
    vmax = np.abs(qkv[:, (nh + kvh) * hd:]).max()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-3 * vmax)


@pytest.mark.parametrize("hd,nh,kvh", [(128, 4, 2), (256, 4, 2), (256, 8, 2), (512, 4, 1), (512, 2, 1)])
@pytest.mark.parametrize("window", [None, 0, 5, 100])
@pytest.mark.parametrize("scale", [0.05, 0.6])
def test_f16_attention_matches_oracle(lib, hd, nh, kvh, window, scale):
    """FP16 operands (impl 3): inputs on the FP16 grid, so the scores are
    exact up to FP32 accumulation and P carries 2^-11 relative rounding; the
    tolerance is the TF32 kernels' 4e-3 relative to the largest |v|."""
    rng = np.random.default_rng(hd * 11 + nh + int(scale * 10))
    lens = [1, 7, 130, 300]
    qkv = rng.standard_normal((sum(lens), (nh + 2 * kvh) * hd), dtype=np.float32) * scale
    qkv = qkv.astype(np.float16).astype(np.float32)
    got, cu = _attention(lib, qkv, lens, nh, kvh, hd, window, 3)
    ref = _attention_ref(qkv, lens, cu, nh, kvh, hd, window)
    assert np.isfinite(got).all()
    vmax = np.abs(qkv[:, (nh + kvh) * hd:]).max()
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-3 * vmax)


def test_f16_attention_rejects_unsupported_shapes(lib):
    """Odd query-head groups and head dims outside {128, 256, 512} are refused
    (the model then keeps the TF32 kernels)."""
    rng = np.random.default_rng(3)
    for hd, nh, kvh in [(256, 3, 1), (64, 2, 1), (192, 4, 2)]:
        lens = [5]
        qkv = rng.standard_normal((5, (nh + 2 * kvh) * hd), dtype=np.float32)
        cu = np.array([0, 5], np.uint64)
        d_qkv = torch.from_numpy(qkv).cuda()
        d_cu = torch.from_numpy(cu.astype(np.int64)).cuda()
        out = torch.empty((5, nh * hd), device="cuda")
        rc = lib.svl_test_attention(d_qkv.data_ptr(), qkv.shape[1], 5, nh, kvh, hd, d_cu.data_ptr(), cu.ctypes.data,
                                    1, -1, 3, out.data_ptr(), nh * hd, None)
        assert rc == 5, (hd, nh, kvh, rc)  # SVL_UNSUPPORTED
