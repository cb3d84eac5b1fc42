"""GPU: sb_gemm_q4_noalloc, the fused int4 GEMM for callers that cannot allocate.

Those callers (a host that reaches the GPU only through the C ABI with no CUDA
allocator of its own, or a process whose device memory is reserved up front by
its own pool) get the split-K scratch from a static device array inside the
library instead of a workspace they pass.  This test calls the new entry point
through the C ABI twice in a row and checks each result against the existing
entry point, sb_gemm_q4 with a caller workspace: bit for bit, since both run
the same kernels with the same split order.  Each result is also held to the
matmul tolerance against the float64 product of the dequantised weight (the
oracle).  It lives in its own file, collected last, and must pass both on its
own in a fresh process and after the other tests.
"""
import numpy as np
import pytest
import torch

from oracle import q4
from slang_b200 import _lib, kernels, synth
from tests._util import assert_close

pytestmark = pytest.mark.gpu


def _noalloc(A, P, S, C, M, N, K):
    lib = _lib.load()
    rc = lib.sb_gemm_q4_noalloc(A.data_ptr(), P.data_ptr(), S.data_ptr(), _lib.SB_F16, 32, C.data_ptr(),
                                M, N, K, 1.0, K, N, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SB_OK, lib.sb_last_error().decode()


# down at M=256 splits K beyond the splits a cluster reduces in distributed
# shared memory, so it takes the static scratch (asserted below); o / k split K
# inside a cluster (no scratch); gate fills the GPU without splitting
CASES = [("down", 256), ("o", 1024), ("k", 512), ("gate", 128), ("gate", 1024)]


@pytest.mark.parametrize("name,M", CASES)
def test_noalloc_matches_workspace_entry_point(cuda, name, M):
    N, K = synth.E2B_SHAPES[name]
    if (name, M) == ("down", 256):
        assert kernels.gemm_q4_workspace_size(M, N, K) > 0, "this case must exercise the static scratch"
    rng = np.random.default_rng(M + N)
    packed, scales = synth.q4_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    A = torch.from_numpy(a).to(cuda)
    P = torch.from_numpy(packed).to(cuda)
    S = torch.from_numpy(scales).to(cuda)
    ws_bytes = kernels.gemm_q4_workspace_size(M, N, K)
    ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=cuda)
    ref = kernels.gemm_q4(A, P, S, workspace=ws).cpu().numpy()
    c64 = q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4))
    for call in range(2):  # two calls in a row share (and reuse) the static scratch
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
        _noalloc(A, P, S, C, M, N, K)
        torch.cuda.synchronize()
        got = C.cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16),
                                      err_msg=f"noalloc {name} M={M} call {call}: not bit-identical to sb_gemm_q4")
        assert_close(got.astype(np.float32), c64, what=f"noalloc {name} M={M} call {call} vs f64 oracle")
    kernels.device_status()
