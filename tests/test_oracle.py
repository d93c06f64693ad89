"""Pin the CPU oracle before trusting it.

The oracle (oracle/fft_oracle.c + oracle/oracle.py) restates the reference's
arithmetic.  Here it is checked against:
  * golden vectors produced by running the reference itself
    (tests/golden/make_golden.py, Triton interpreter on CPU);
  * the reference's own C++ FFT compiled in place (oracle/_ref), when built;
  * the known answers of the reference's tests (bitrev(8), impulse, tone,
    naive DFT at N = 8..4096 as in src/host/fft_check.cpp).
"""
import numpy as np
import pytest

from oracle import oracle as O

from conftest import cplx

# Oracle vs the reference's own FP32 outputs: both compute the same stage
# cascades in float32; they differ only in twiddle rounding (float32 angles in
# the reference), measured <= 3e-7 relative L2.
TOL_VS_REF = 1e-6


@pytest.mark.parametrize("kind", ["bitrev", "dit_digrev", "dif_digrev"])
def test_index_maps_bit_exact_vs_reference_kernels(golden, kind):
    for bits in range(1, 13):
        np.testing.assert_array_equal(O.index_table(kind, bits), golden[f"idx_{kind}_{bits}"])


def test_bitrev_known_answer():
    # src/host/fft_check.cpp:43-54
    assert list(O.index_table("bitrev", 3)) == [0, 4, 2, 6, 1, 5, 3, 7]


def test_bitrev_permute_vs_reference(golden):
    for n in (8, 64, 1024):
        x = np.arange(n, dtype=np.float32).astype(np.complex64)
        np.testing.assert_array_equal(O.bitrev_permute(x), golden[f"bitrev_permute_{n}"])


def _oracle_for_case(c, x):
    r = c.get("runner")
    if "plan" in c:
        p = c["plan"]
        return O.execute(p["executed"], x, p["transform_type"], p["transform_direction"], p["norm"],
                         p["params"].get("real_flow"), p["params"])
    if r == "r2c_stitch":
        return O.r2c_stitch(x, c["n"], c["scale"])
    if r == "c2r_pre":
        return O.c2r_pre(x, c["n"])
    if r == "c2r_unpack":
        return O.c2r_unpack(x, c["n"], c["scale"])
    return O.core_fft(r, x, c)


def test_oracle_matches_every_reference_golden_case(golden, golden_meta):
    worst = {}
    for c in golden_meta["cases"]:
        lab = c["label"]
        got = _oracle_for_case(c, golden[lab + "__in"])
        e = O.rel_l2(got, golden[lab + "__out"])
        worst[lab] = e
        assert e <= TOL_VS_REF, (lab, e)
    assert len(worst) >= 50


def test_exact_cases_are_bit_exact(golden):
    # permutation-only / trivial-twiddle paths reproduce the reference bit for bit
    for lab in ("fft_dit_2", "fft_dit_radix4_4", "fft_dif_radix4_4", "fft_dit_radix4_8",
                "fft_dif_radix4_8", "c2r_unpack_64x3", "c2r_unpack_1024x2", "kat_impulse_256",
                "kat_const34_256"):
        x, y = golden[lab + "__in"], golden[lab + "__out"]
        if lab.startswith("c2r_unpack"):
            n = y.shape[-1]
            got = O.c2r_unpack(x, n, 0.25)
        else:
            got = O.core_fft("fft_dit_radix4" if "radix4" in lab else
                             ("fft_dif_radix4" if "dif_radix4" in lab else "fft_dit"), x)
            if "dif_radix4" in lab:
                got = O.fft_radix4_f32(x, dif=True)
        np.testing.assert_array_equal(got.view(np.uint8), y.astype(got.dtype).view(np.uint8), err_msg=lab)


def test_known_signals(golden):
    n = 256
    imp = golden["kat_impulse_256__out"]
    np.testing.assert_allclose(imp, np.ones(n), atol=1e-6)
    tone = golden["kat_tone5_256__out"]
    ref = np.zeros(n, np.complex128)
    ref[5] = n
    assert O.rel_l2(tone, ref) < 1e-6
    assert O.rel_l2(O.fft_radix2_f32(golden["kat_tone5_256__in"]), ref) < 1e-6


@pytest.mark.parametrize("n", [8, 16, 64, 256, 1024, 4096])
@pytest.mark.parametrize("dif", [False, True])
def test_f64_path_vs_naive_dft(n, dif):
    # src/host/fft_check.cpp:57-77: deterministic input, naive DFT, rel < 1e-10
    i = np.arange(n)
    x = np.sin(0.1 * i + 1.3) + 1j * np.cos(0.2 * i + 0.7)
    k = np.arange(n)
    ref = np.exp(-2j * np.pi * np.outer(k, i) / n) @ x
    got = O.fft_f64(x, dif=dif)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-10


def test_f64_vs_numpy_and_inverse():
    rng = np.random.default_rng(7)
    x = cplx(rng, (3, 512)).astype(np.complex128)
    np.testing.assert_allclose(O.fft_f64(x), np.fft.fft(x), rtol=0, atol=1e-9)
    np.testing.assert_allclose(O.fft_f64(x, inverse=True) / 512, np.fft.ifft(x), atol=1e-12)


def test_reference_cpp_fft_pins_the_f64_restatement():
    L = O.reference_lib()
    if L is None:
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    assert [L.ref_bit_reverse(i, 3) for i in range(8)] == [0, 4, 2, 6, 1, 5, 3, 7]
    rng = np.random.default_rng(11)
    for n in (8, 256, 4096):
        x = cplx(rng, (4, n)).astype(np.complex128)
        for dif in (False, True):
            ref = O.reference_fft_c128(x, dif=dif, threads=2)
            np.testing.assert_allclose(O.fft_f64(x, dif=dif), ref, rtol=0, atol=1e-10 * np.sqrt(n))


def test_radix4_and_radix2_agree_with_numpy():
    rng = np.random.default_rng(3)
    for n in (4, 8, 32, 128, 2048):
        x = cplx(rng, (2, n))
        ref = np.fft.fft(x.astype(np.complex128))
        for fn in (O.fft_radix2_f32, O.fft_radix4_f32):
            for dif in (False, True):
                assert O.rel_l2(fn(x, dif=dif), ref) < 1e-6


def test_real_epilogues_compose_to_rfft_irfft():
    rng = np.random.default_rng(5)
    n, b = 64, 3
    x = rng.standard_normal((b, n)).astype(np.float32)
    z = x.view(np.complex64)
    got = O.r2c_stitch(O.fft_radix2_f32(z), n)
    assert O.rel_l2(got, np.fft.rfft(x.astype(np.float64))) < 1e-6
    xh = np.fft.rfft(x.astype(np.float64)).astype(np.complex64)
    back = O.c2r_unpack(O.fft_radix2_f32(O.c2r_pre(xh, n)), n, 2.0 / n)
    assert O.rel_l2(back, x) < 1e-6


def test_local_matrix_is_the_tile_dft_on_bitreversed_input():
    # src/xpu/matrices.py:64-92 contract: DIT local group on a bit-reversed tile == DFT
    for tile in (8, 32, 64):
        m = O.local_matrix(tile, "dit")
        perm = O.index_table("bitrev", tile.bit_length() - 1)
        dft = np.exp(-2j * np.pi * np.outer(np.arange(tile), np.arange(tile)) / tile)
        np.testing.assert_allclose(m, dft[:, perm], atol=1e-12)
        md = O.local_matrix(tile, "dif")
        np.testing.assert_allclose(md, dft[perm, :], atol=1e-12)


def test_hybrid_restatement_is_a_dft():
    rng = np.random.default_rng(9)
    x = cplx(rng, (2, 1024))
    for tile in (32, 64):
        assert O.rel_l2(O.hybrid_4step(x, tile), np.fft.fft(x.astype(np.complex128))) < 1e-6


def test_rel_l2_is_nan_safe():
    assert O.rel_l2(np.array([np.nan]), np.array([1.0])) == float("inf")


def test_oracle_matches_the_reference_rows_at_baseline_shapes():
    """The row-subset fixture (the reference's output on the first rows of
    configurations 2, 3, 4 and 5a, tests/golden/make_golden_rows.py) pins the
    oracle at the BASELINE shapes too; the fixture itself is a transform
    (float64 check at its sampled positions)."""
    import json
    import os

    from conftest import GOLDEN_DIR
    from golden import row_cases

    with open(os.path.join(GOLDEN_DIR, "reference_rows.json")) as f:
        meta = json.load(f)["cases"]
    rows = np.load(os.path.join(GOLDEN_DIR, "reference_rows.npz"))
    assert {m["config"] for m in meta.values()} >= {"2", "3", "4", "5a"}
    for case in row_cases.CASES:
        lab = case["label"]
        if lab not in meta:
            continue
        x = row_cases.case_input(case)
        pos, want = rows[lab + "__pos"], rows[lab + "__out"]
        if case["ref"] == "plan":
            got = O.execute(case["executed"], x, case["tt"], case["td"], "backward",
                            case["params"].get("real_flow"), case["params"])
        else:
            got = O.core_fft(case["ref"], x, case["knobs"])
        assert list(got.shape) == meta[lab]["out_shape"], lab
        e = O.rel_l2(got.reshape(-1)[pos], want)
        assert e <= TOL_VS_REF, (lab, e)
        if case["tt"] == "c2c":
            x64 = x.astype(np.complex128)
            ref64 = np.fft.fft(x64, axis=-1) if case["td"] == "forward" else np.fft.ifft(x64, axis=-1)
        elif case["tt"] == "r2c":
            ref64 = np.fft.rfft(x.astype(np.float64), axis=-1)
        else:
            ref64 = np.fft.irfft(x.astype(np.complex128), n=case["n"], axis=-1)
        assert O.rel_l2(want, ref64.reshape(-1)[pos]) <= 1e-6, lab
