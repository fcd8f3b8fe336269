"""Failure handling on the GPU without faulting it: a bounded device wait
that runs out reports WATTN_ERR_TIMEOUT and leaves the context usable, and
bad arguments are rejected before any launch."""
import numpy as np
import pytest

from tests.helpers import check_f32, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def test_bounded_wait_reports_timeout_and_device_survives(W, oracle):
    import torch
    torch.cuda.synchronize()
    assert W.device_status() == 0
    assert W.selftest_bounded_wait(2000) == -4      # a flag nothing sets: 2 ms limit
    assert W.device_status() == 0                  # read and cleared by the self-test
    # the context is still usable: run a real kernel and check it
    h, d, t = 2, 128, 100
    q, k, v = randn(1, t * d), randn(2, t * d), randn(3, t * d)
    out = np.empty_like(q)
    W.flash_attention_2(q, k, v, t, t, h, d, False, out)
    check_f32(out, oracle.flash_attention_2(q, k, v, t, t, h, d, False), "after timeout")


def test_misaligned_and_bad_arguments_rejected(W):
    import torch
    x = torch.zeros(4096, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros(4096, dtype=torch.float32, device="cuda")
    with pytest.raises(W.WattnError) as e:   # q one element off a 16-byte boundary
        W.attention_fwd(x[1:], x, x, o, batch=1, t_q=8, t_kv=8, n_heads=2, scale=0.125)
    assert e.value.status == -1
    with pytest.raises(W.WattnError) as e:   # row stride not a multiple of 16 bytes
        W.attention_fwd(x, x, x, o, batch=1, t_q=8, t_kv=8, n_heads=2, scale=0.125,
                        q_row_stride=130)
    assert e.value.status == -1
    with pytest.raises(W.WattnError) as e:   # f16 input with bf16 output
        W.attention_fwd(x.view(torch.float16), x.view(torch.float16), x.view(torch.float16),
                        x, batch=1, t_q=8, t_kv=8, n_heads=2, scale=0.125)
    assert e.value.status == -1
    with pytest.raises(W.WattnError):        # too small a workspace
        W.decode_fwd(x, x, x, o, n_groups=2, group_size=2, t_kv=1000, n_heads=1, scale=0.125,
                     workspace=torch.zeros(16, dtype=torch.uint8, device="cuda"))
    torch.cuda.synchronize()
    assert W.device_status() == 0
