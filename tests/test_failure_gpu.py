"""Failure detection without a GPU fault: a kernel whose mbarrier wait can never complete gives up
after a short wall-clock limit, records a status bit and returns; the context stays usable."""
import numpy as np
import pytest

import gpt2_b200 as G
import oracle as O
from conftest import assert_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives(cuda, lib, oracle):
    assert lib.status(clear=True) == 0
    rc = lib.gpt2_b200_selftest_wait_timeout(20000)  # 20 ms limit on a wait nothing satisfies
    assert rc == G.ETIMEOUT
    assert lib.status() == 0  # the self-test consumed its own bit
    T = 130
    x = O.seeded_qkv(130, T)
    att = cuda.empty((T, O.E), dtype=cuda.float16, device="cuda")
    lib.prefill(att, cuda.from_numpy(x.astype(np.float16)).cuda(), T)
    cuda.cuda.synchronize()
    assert_close(att.float().cpu().numpy(), oracle.prefill(x), "prefill after the timeout test")
