"""GPU: the tensor-core operand encodings (descriptors, instruction descriptor, TMEM layout,
shifted A rows, collector reuse) checked on one CTA against a CPU matmul before anything larger
trusts them."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [16, 32, 48, 64])
@pytest.mark.parametrize("shift", [0, 1, 2])
@pytest.mark.parametrize("collector", [0, 1])
def test_umma_encodings(n, shift, collector):
    import ajib
    rng = np.random.default_rng(1000 + n * 10 + shift)
    a = rng.uniform(-1, 1, size=(130, 32)).astype(np.float16)
    b = rng.uniform(-1, 1, size=(2 * n, 32)).astype(np.float16)
    da = torch.from_numpy(a).cuda()
    db = torch.from_numpy(b).cuda()
    out = torch.zeros((2, 128, n), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = ajib.lib.ajib_selftest_umma(da.data_ptr(), db.data_ptr(), out.data_ptr(), n, shift, collector,
                                     err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "the self-test's wait timed out"
    af = a.astype(np.float32)[shift:shift + 128]
    bf = b.astype(np.float32)
    want = np.stack([af @ bf[:n].T, af @ bf[n:].T])
    got = out.cpu().numpy()
    assert np.abs(got - want).max() < 1e-3
