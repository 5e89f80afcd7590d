"""Properties of the arithmetic the oracle and the kernels share (CPU only)."""
import numpy as np
import torch


def ulp_diff(a, b):
    a = a.astype(np.float32).view(np.int32).astype(np.int64)
    b = b.astype(np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, np.int64(-2**31) - a, a)
    b = np.where(b < 0, np.int64(-2**31) - b, b)
    return np.abs(a - b)


def test_expf_accuracy(oracle):
    # Cody-Waite + degree-7 Taylor: within 2 ulp of float64 exp over the whole finite range
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-103.9, 88.7, 200000), rng.uniform(-2, 2, 200000),
                        np.array([0.0, -0.0, 1.0, -1.0, 88.72, -87.3, -100.0], np.float64)]).astype(np.float32)
    got = oracle.expf(x)
    ref = np.exp(x.astype(np.float64)).astype(np.float32)
    normal = ref >= np.finfo(np.float32).tiny
    assert ulp_diff(got[normal], ref[normal]).max() <= 2
    assert np.all(np.abs(got[~normal] - ref[~normal]) <= 2 * 2.0 ** -149 * 8)
    assert oracle.expf(np.array([100.0, -200.0], np.float32)).tolist() == [np.inf, 0.0]


def test_gelu_matches_torch_tanh_gelu(oracle):
    x = np.linspace(-12, 12, 100001).astype(np.float32)
    got = oracle.gelu_tanh(x)
    ref = torch.nn.functional.gelu(torch.from_numpy(x).double(), approximate="tanh").numpy()
    assert np.max(np.abs(got - ref)) < 2e-6 * max(1.0, np.abs(ref).max())


def test_int8_partial_fits_exact_conversion():
    # |sum of 128 int8 x int8 products| <= 128 * 127^2 = 2,064,512 < 2^22, so the kernels' integer ->
    # float conversion (add 0x4B400000 to the int32, reinterpret, subtract 1.5 * 2^23) is exact.
    assert 128 * 127 * 127 < 2 ** 22
    p = np.arange(-2 ** 22, 2 ** 22, dtype=np.int64)
    f = ((p + 0x4B400000).astype(np.uint32)).view(np.float32) - np.float32(12582912.0)
    assert np.array_equal(f.astype(np.float64), p.astype(np.float64))


def test_e4m3_conversion_matches_torch(oracle):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(100000) * 100, rng.standard_normal(10000) * 1e-2,
                        np.array([448.0, -448.0, 447.9, 0.0, -0.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10])])
    x = np.clip(x, -448, 448).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    q, _ = oracle.quantize_activations(np.ones((1, 128), np.float32) * 448.0, "fp8")
    assert q[0, 0] == 0x7E   # 448 / (448 / 448) -> max normal
    import ctypes
    got = np.array([oracle.lib().or_e4m3_from_f32(ctypes.c_float(v)) for v in x[:20000]], dtype=np.uint8)
    assert np.array_equal(got, ref[:20000])


def tie_rows():
    """Rows whose scale is exactly 1 (absmax 127) and whose other values are exact ties k + 0.5, all bf16."""
    ties = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 3.5, 126.5, -126.5, 0.25, 3.75]
    row = np.zeros(128, dtype=np.float32)
    row[0] = 127.0
    row[1:1 + len(ties)] = ties
    return np.stack([row, -row]), ties


def test_round_half_even_option_on_ties(oracle):
    """Per-token and per-group int8 codes on exact ties: half away from zero (the reference) and half to even
    (the option beside it)."""
    x, ties = tie_rows()
    away = {0.5: 1, 1.5: 2, 2.5: 3, 3.5: 4, 126.5: 127, 0.25: 0, 3.75: 4}
    even = {0.5: 0, 1.5: 2, 2.5: 2, 3.5: 4, 126.5: 126, 0.25: 0, 3.75: 4}
    for per_row in (False, True):
        for rne, table in ((False, away), (True, even)):
            q, s = oracle.quantize_activations(x, "int8", per_row=per_row, round_half_even=rne)
            assert np.all(s == 1.0)
            codes = q.view(np.int8)
            for i, t in enumerate(ties):
                want = int(np.sign(t)) * table[abs(t)]
                assert codes[0, 1 + i] == want and codes[1, 1 + i] == -want, (per_row, rne, t)
