"""The bounded waits of the peer-memory expert exchange, made to run out on one GPU.

A world-2 mailbox lives on the local GPU and no peer ever dispatches into it, so the dispatch
and return flags never arrive. With a short poll limit each wait gives up on its own: the
kernel sets the error word (state[3]), marks every received slot as the dummy expert and
returns, the context stays usable, and the host-side checks of the exchange and of the MoE
decoder raise. Nothing waits on another kernel: the flag is simply never written."""
from __future__ import annotations

import ctypes
import types

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_p2p_waits_time_out_and_report(cuda):
    from mrun_b200 import _lib
    from mrun_b200.expert_parallel import P2PExpertParallelMoE
    from mrun_b200.moe_engine import MoeDecoder

    lib = _lib.load()
    world, cap, hidden, dummy = 2, 8, 256, 4
    nbytes = int(lib.mrb_ep_mailbox_bytes(world, cap, hidden))
    own = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    _lib.call("mrb_ep_mailbox_create", nbytes, ctypes.byref(own), handle)
    default = int(lib.mrb_ep_wait_limit())
    assert default == 1 << 22
    try:
        _lib.call("mrb_ep_set_wait_limit", 2000)  # about 0.1-1 ms per wait
        assert int(lib.mrb_ep_wait_limit()) == 2000
        stream = _lib.stream_handle(cuda)
        state = torch.tensor([7, 0, 0, 0], dtype=torch.int32, device=cuda)  # epoch 7: never published
        ids64 = torch.full((world * cap,), -5, dtype=torch.int64, device=cuda)
        _lib.call("mrb_ep_p2p_wait_dispatch", own.value, world, cap, hidden, dummy, ids64.data_ptr(),
                  state.data_ptr(), stream)
        torch.cuda.synchronize(cuda)
        assert int(state[3]) == 1
        assert torch.equal(ids64.cpu(), torch.full((world * cap,), dummy, dtype=torch.int64))
        state[3] = 0
        _lib.call("mrb_ep_p2p_wait_return", own.value, world, cap, hidden, state.data_ptr(), stream)
        torch.cuda.synchronize(cuda)
        assert int(state[3]) == 1
        # the context is still usable after the waits gave up
        x = torch.arange(16, device=cuda, dtype=torch.float32)
        assert float(x.sum()) == 120.0
        # host-side reporting: the exchange's check and the decoder's check both raise
        exchange = types.SimpleNamespace(state=state)
        with pytest.raises(RuntimeError, match="timed out"):
            P2PExpertParallelMoE.check(exchange)
        decoder = types.SimpleNamespace(error_flag=torch.zeros(1, dtype=torch.int32, device=cuda),
                                        ep=[types.SimpleNamespace(check=lambda: P2PExpertParallelMoE.check(exchange))])
        with pytest.raises(RuntimeError, match="timed out"):
            MoeDecoder.check_errors(decoder)
    finally:
        _lib.call("mrb_ep_set_wait_limit", default)
        torch.cuda.synchronize(cuda)
        _lib.call("mrb_ep_mailbox_close", own.value, 1)

