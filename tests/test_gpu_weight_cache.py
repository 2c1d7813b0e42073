"""GPU: a weight written to the repacked-weight cache and opened again is the same weight: its
exported MLX arrays are bit-identical, its scale flags are recomputed, and its matmuls give the
same bits as the original handle's."""
import pytest
import torch

from gpu_util import u16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("large_scales", [False, True])
def test_cache_round_trip(cuda, oracle, tmp_path, large_scales):
    from helios_b200 import quantized as Q
    N, K = 4096, 3840
    w, s, b = Q.synth_matrix(oracle.matrix_seed(12, oracle.PROJ_IDS["q"]), N, K)
    if large_scales:   # |scale| >= 2^-1 on some rows: the kernels must leave the raw odd-nibble form
        s = s.clone()
        s[::97] = 0.75
    qw = Q.QuantizedWeight.from_mlx(w, s, b)
    path = tmp_path / "q.g4qc"
    qw.save(path)
    assert path.stat().st_size == 64 + N * K // 2 + N * (K // 64) * 4
    qo = Q.QuantizedWeight.open(path)
    assert qo.shape == (N, K) and qo.info()["fast_path_ok"] == qw.info()["fast_path_ok"] == 1
    for a, c in zip(qw.export(), qo.export()):
        assert torch.equal(a.view(torch.int16) if a.dtype != torch.uint32 else a.view(torch.int32),
                           c.view(torch.int16) if c.dtype != torch.uint32 else c.view(torch.int32))
    for M in (1, 4, 64):
        x = Q.synth_normal(oracle.activation_seed(90 + M), (M, K))
        y0, y1 = Q.quantized_matmul(x, qw), Q.quantized_matmul(x, qo)
        torch.cuda.synchronize()
        assert (u16(y0) == u16(y1)).all()
    qw.free()
    qo.free()
