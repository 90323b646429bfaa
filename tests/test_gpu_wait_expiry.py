"""Error path of the bounded device waits, on the B200, without a GPU fault.

The reference's host loop treats a PL that reports an error, or does not
finish in time, as fatal for the request (src/software/generation.c:21-25:
the -3 and -2 returns; main.c:270-273 resets the context). Every spin and
mbarrier wait of this library's kernels is bounded: when a wait runs out the
kernel records a code in a device error flag and returns normally, and the
host reports it. qwen_b200_test_expire_wait makes one such wait run out on
purpose: the last grid barrier of the persistent single-row step waits for one
arrival more than its CTAs make, with a short limit, at a point where no bulk
copy or tensor-core operation is in flight. The tests check that the call
reports QWEN_B200_ETIMEOUT (CSR status 8 with error code 5 through the
qgen_ops protocol), that nothing advances, and that the same handle computes
the right tokens afterwards.
"""
import ctypes

import numpy as np
import pytest

import qwen_b200
from qwen_b200 import _lib
from qgen import EngineOps, qgen_run

pytestmark = pytest.mark.gpu
L = qwen_b200.lib


@pytest.fixture(scope='module')
def engine(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=1, max_context=64, max_rows=64).load_assets(sd_root)
    yield e
    L().qwen_b200_test_expire_wait(e.h, 0)
    e.close()


def test_expired_barrier_reports_timeout_and_the_handle_recovers(engine, golden):
    prompt = list(golden['prompt'])
    engine.reset(0)
    first, _ = engine.forward(0, prompt, 0)
    second, _ = engine.forward(0, [first], len(prompt))  # the persistent step, switch off
    engine.reset(0)
    assert engine.forward(0, prompt, 0)[0] == first
    assert L().qwen_b200_test_expire_wait(engine.h, 1) == 0
    ids = np.array([first], np.uint32)
    tok = ctypes.c_uint32(0)
    status = L().qwen_b200_forward(engine.h, 0, ids.ctypes.data_as(_lib._P32), 1, len(prompt), ctypes.byref(tok),
                                   None)
    assert status == _lib.ETIMEOUT, L().qwen_b200_last_error(engine.h)
    assert b'timed out' in L().qwen_b200_last_error(engine.h)
    assert engine.position(0) == len(prompt)  # the failed step did not advance the slot
    assert L().qwen_b200_test_expire_wait(engine.h, 0) == 0
    # the same handle, the same step: the right token, and the flag is clear
    assert engine.forward(0, [first], len(prompt))[0] == second
    assert engine.forward(0, [second], len(prompt) + 1)[0] >= 0


def test_expired_barrier_through_the_csr_protocol(engine, golden):
    prompt = list(golden['prompt'])
    engine.reset(0)
    first, _ = engine.forward(0, prompt, 0)
    second, _ = engine.forward(0, [first], len(prompt))
    ops = EngineOps(L(), engine.h)
    L().qwen_b200_clear(engine.h)
    assert L().qwen_b200_test_expire_wait(engine.h, 1) == 0
    # the prefill (16 rows, per-kernel path) finishes; the first decode step
    # (one row, persistent path) reports the expired wait as a PL error
    status, res, toks = qgen_run(ops, prompt, 3)
    assert status == -3 and res.produced == 1 and toks == [first]
    assert L().qwen_b200_csr_read(engine.h, 0x18) == 8
    assert L().qwen_b200_csr_read(engine.h, 0x30) == 5
    # as main.c:270-273 does after a PL error: reset the context, run again
    assert L().qwen_b200_test_expire_wait(engine.h, 0) == 0
    L().qwen_b200_clear(engine.h)
    status, res, toks = qgen_run(ops, prompt, 2)
    assert status == 0 and toks == [first, second]
