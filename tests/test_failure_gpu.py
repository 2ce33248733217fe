"""Failure detection on the device without a GPU fault: a bounded wait that
runs out (on an mbarrier nothing arrives on) records its site code in an error
word, the host reads KB200_ERR_TIMEOUT, and the context stays usable -- the next
kernels run and give correct results.  The status query of the GDN op reports
OK after a normal call."""
import ctypes

import pytest
import torch

from kairos_sensenova_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_timeout():
    L = _lib.lib()
    word = torch.zeros(4, dtype=torch.int32, device='cuda')
    st = torch.cuda.current_stream().cuda_stream
    # ~1e6 SM clocks (well under a millisecond): the wait gives up, the kernel returns
    assert L.kb200_wait_probe(word.data_ptr(), 1_000_000, st) == 0
    assert L.kb200_read_error_word(word.data_ptr(), st) == _lib.ERRORS_BY_NAME['timeout']
    assert b'site 99' in L.kb200_last_error()
    assert int(word[0]) == 99
    # the context is still usable: a normal GDN call afterwards runs and reports OK
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    gen = torch.Generator(device='cuda').manual_seed(0)
    q, k, v = (torch.randn(1, 200, 2, 128, generator=gen, device='cuda').bfloat16() for _ in range(3))
    g = -torch.rand(1, 200, 2, generator=gen, device='cuda')
    beta = torch.rand(1, 200, 2, generator=gen, device='cuda').bfloat16()
    o, s = chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True,
                                  check=True)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(s).all()
    word.zero_()
    assert L.kb200_read_error_word(word.data_ptr(), st) == 0
