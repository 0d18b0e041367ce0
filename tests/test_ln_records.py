"""The arithmetic of the fused LayerNorm's statistics, on CPU: the segment records that the GEMM epilogue
and row_seg_stats write (dev.cuh seg_add / seg_record: fp32, shifted by the segment's first value, even
and odd columns in separate lanes) and their combination per row (ln_from_records: the mean of the
segment means, then M2 = sum of (M2_s + segw (mean_s - mean)^2)), restated operation by operation in
numpy float32, against float64 two-pass statistics of the same fp16 rows. Rows with means of up to
10^3 standard deviations: the shift keeps the sums free of cancellation. The device code itself is
checked against float64 on a B200 (tests/test_kernels_gpu.py::test_gemm_ln_records)."""
import numpy as np
import pytest

f32 = np.float32


def fma32(a, b, c):
    return f32(np.float64(a) * np.float64(b) + np.float64(c))


def seg_record(x, segw):
    """{mean, M2} of one segment, in the device's order of fp32 operations."""
    k = f32(x[0])
    s1 = [f32(0), f32(0)]
    s2 = [f32(0), f32(0)]
    for j in range(segw):
        d = f32(f32(x[j]) - k)
        s1[j & 1] = f32(s1[j & 1] + d)
        s2[j & 1] = fma32(d, d, s2[j & 1])
    a = f32(s1[0] + s1[1])
    q = f32(s2[0] + s2[1])
    m = f32(a / f32(segw))
    return f32(k + m), fma32(-a, m, q)


def ln_from_records(recs, segw, eps):
    ms = f32(0)
    for r in recs:
        ms = f32(ms + r[0])
    mean = f32(ms / f32(len(recs)))
    m2 = f32(0)
    for r in recs:
        dm = f32(r[0] - mean)
        m2 = f32(m2 + fma32(f32(f32(segw) * dm), dm, r[1]))
    var = f32(m2 / f32(f32(segw) * f32(len(recs))))
    return mean, f32(1.0) / f32(np.sqrt(f32(var + f32(eps))))


@pytest.mark.parametrize("C,segw", [(128, 64), (384, 128), (1024, 128), (2048, 128)])
@pytest.mark.parametrize("shift", [0.0, 3.0, 30.0, 1000.0])
def test_records_match_two_pass_statistics(C, segw, shift):
    rng = np.random.default_rng(C + int(shift))
    rows = (rng.normal(size=(6, C)) * rng.uniform(0.5, 2.0, size=(6, 1)) + shift).astype(np.float16)
    for x in rows:
        recs = [seg_record(x[s:s + segw], segw) for s in range(0, C, segw)]
        mean, rstd = ln_from_records(recs, segw, 1e-5)
        xd = x.astype(np.float64)
        m64 = xd.mean()
        v64 = ((xd - m64) ** 2).mean()
        r64 = 1.0 / np.sqrt(v64 + 1e-5)
        assert abs(float(mean) - m64) <= 2e-7 * (abs(m64) + np.sqrt(v64))
        assert abs(float(rstd) - r64) <= 1e-5 * r64
