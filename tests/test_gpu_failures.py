"""Failure detection on the GPU without faulting it: a device wait that runs out is reported as BCU_ERR_TIMEOUT and
the context stays usable; a cancel raised by another host thread stops a decode between steps (the reference's stop
flag, ext.rs:21-42) with BCU_ERR_CANCELLED, and the model works afterwards."""
import threading
import time

import numpy as np
import pytest

from bonsai_b200 import _lib, synth
from bonsai_b200.config import tiny
from bonsai_b200.runtime import BackendError, Model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(gpu):
    cfg = tiny(ctx=16384)
    m = Model(cfg).load(synth.model_tensors(cfg, 17))
    yield cfg, m
    m.close()


def test_device_wait_timeout_is_reported(model):
    cfg, m = model
    ids = synth.zipf_tokens(1, 20, cfg.vocab)
    m.reset()
    want = m.prefill(ids)
    st, msg = m.debug_wait_timeout()
    assert st == _lib.ERR_TIMEOUT and "gave up" in msg
    # the error was read and cleared; the context still runs the model, with the same result
    m.reset()
    assert m.prefill(ids) == want
    assert m.debug_wait_timeout()[0] == _lib.ERR_TIMEOUT  # and reports again


@pytest.mark.parametrize("speculate", [False, True])
def test_cancel_from_another_thread(model, speculate):
    cfg, m = model
    ids = synth.zipf_tokens(2, 32, cfg.vocab)
    m.reset()
    first = m.prefill(ids)
    result = {}

    def run():
        try:
            out, _ = m.decode(first, user=ids, speculate=speculate, max_tokens=16000)
            result["n"] = len(out)
        except BackendError as e:
            result["status"] = e.status

    th = threading.Thread(target=run)
    th.start()
    time.sleep(0.05)
    m.cancel(True)
    th.join(60)
    assert not th.is_alive()
    assert result.get("status") == _lib.ERR_CANCELLED, result
    m.cancel(False)
    m.reset()
    assert m.prefill(ids) == first  # usable afterwards
