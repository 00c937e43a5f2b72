"""The five BASELINE workloads at full size against the FP64 C oracle.

Gate: FP16 inputs max-abs 2e-3 / rel 1e-3, FP32 inputs
1e-5, applied as assert_allclose(atol, rtol).  The oracle runs on the same
tensors copied to the host, threaded over all host cores.  The observed max
abs error of every config is printed.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("NVIDIA GPU required", allow_module_level=True)

from oracle import c_oracle
from paged_decode import workload
from paged_decode.runtime import DecodePlan

pytestmark = pytest.mark.gpu

TOL = {"float16": dict(atol=2e-3, rtol=1e-3), "float32": dict(atol=1e-5, rtol=1e-5)}


@pytest.mark.parametrize("name", ["c1", "c2", "c3a", "c3b", "c3c", "c4", "c5"])
def test_baseline_config_matches_oracle(name):
    w = workload.CONFIGS[name]()
    q, k, v = w.tensors("cuda")
    plan = DecodePlan(w.layout, w.table, w.lengths, split_tokens=w.split_tokens)
    out = plan.run(q, k, v).cpu().numpy()
    assert plan.read_errors() == 0
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))
    del q, k, v
    torch.cuda.empty_cache()
    ref = c_oracle.dense_attention(qh, kh, vh, w.table, w.lengths, threads=os.cpu_count())
    err = float(np.abs(out - ref).max())
    print(f"{w.name}: max abs err {err:.3e}")
    np.testing.assert_allclose(out, ref, **TOL[w.dtype])
