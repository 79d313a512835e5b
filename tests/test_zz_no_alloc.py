"""The allocation-free GEMM entry point (needs a B200).

jal_cached_matrix_gemm_noalloc exists for callers that cannot allocate device
memory while they run: a process whose free device memory already belongs to
another allocator's pool, or a serving loop that must not call
cudaMalloc/cudaFree because they can synchronise the whole device.  It keeps
the quantized activations in a fixed 2 MiB device array instead of a per-call
buffer.  These tests call it through the C ABI several times in a row on one
stream (so each call runs over what the previous one left in the shared
array) and compare each result with jal_cached_matrix_gemm and with the
oracle's project_batch (repack_cache.rs:1739-1787); all three compute in the
reference's f32 order, so the results must be equal bit for bit.

The file is named so that pytest collects it last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 2 << 20


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("quant_name", ["Q4_0", "Q8_0"])
def test_noalloc_gemm_matches_gemm_and_oracle_on_successive_calls(jal, oracle, torch_cuda, quant_name):
    torch = torch_cuda
    quant = getattr(jal, quant_name)
    rows, cols = 1000, 4096
    raw = jal.synth_matrix(quant, rows, cols, seed=31, name="noalloc")
    mat = jal.CachedMatrix.repack(raw, quant, rows, cols)
    ref_w = oracle.RepackedWeight(raw, quant, rows, cols)
    lib = jal.lib()
    # 40 tokens (tiled GEMM), 1 token (decode GEMV), 3 tokens (GEMM again),
    # each with different activations over the array the previous call filled.
    cases = [(40, jal.synth_normal(40 * cols, seed=32, name="noalloc.a")),
             (1, 3.0 * jal.synth_normal(cols, seed=35, name="noalloc.c")),
             (3, 5.0 * jal.synth_normal(3 * cols, seed=33, name="noalloc.b"))]
    xs = [_dev(torch, x) for _, x in cases]
    outs = [torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda") for m, _ in cases]
    torch.cuda.synchronize()
    for (m, _), x, y in zip(cases, xs, outs):
        rc = lib.jal_cached_matrix_gemm_noalloc(mat._h, x.data_ptr(), m, y.data_ptr(), None)
        assert rc == 0, lib.jal_last_error().decode()
    torch.cuda.synchronize()
    for (m, xh), x, y in zip(cases, xs, outs):
        want = torch.zeros(m * rows, dtype=torch.float32, device="cuda")
        rc = lib.jal_cached_matrix_gemm(mat._h, x.data_ptr(), m, want.data_ptr(), None)
        assert rc == 0, lib.jal_last_error().decode()
        torch.cuda.synchronize()
        got, ref = y.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert np.array_equal(got, ref)
        assert np.array_equal(got.reshape(m, rows), ref_w.project_batch(xh, m, nthreads=8))


def test_noalloc_gemm_rejects_oversize(jal, torch_cuda):
    torch = torch_cuda
    rows, cols = 64, 4096
    raw = jal.synth_matrix(jal.Q4_0, rows, cols, seed=34, name="noalloc.big")
    mat = jal.CachedMatrix.repack(raw, jal.Q4_0, rows, cols)
    # 456 tokens x 4096 cols needs 456*4096 + 456*128*4 bytes > 2 MiB.
    m = 456
    assert m * cols + m * (cols // 32) * 4 > SCRATCH_BYTES
    x = torch.zeros(m * cols, dtype=torch.float32, device="cuda")
    y = torch.full((m * rows,), 7.0, dtype=torch.float32, device="cuda")
    lib = jal.lib()
    rc = lib.jal_cached_matrix_gemm_noalloc(mat._h, x.data_ptr(), m, y.data_ptr(), None)
    assert rc == jal.ERR_TENSOR_BOUNDS
    assert "scratch" in lib.jal_last_error().decode()
    torch.cuda.synchronize()
    assert bool(torch.all(y == 7.0))
    # The largest size that fits still runs.
    m_ok = 455
    rc = lib.jal_cached_matrix_gemm_noalloc(mat._h, x.data_ptr(), m_ok, y.data_ptr(), None)
    assert rc == 0, lib.jal_last_error().decode()
    torch.cuda.synchronize()
