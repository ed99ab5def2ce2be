"""Every device wait is bounded, and a wait that runs out leaves cleanly (no GPU fault, no hang): on the B200,
  * the tensor-parallel reduce on one GPU for 2 ranks with an arrival flag that nothing sets: the call's wait gives up
    after its limit, the context's error word carries the timeout bit, nothing is written, and the context runs the
    next kernel; with the flag set, the same call sums and writes;
  * the fused decode step with its wait limit at zero: waits for other CTAs' work run out at once, the step leaves
    undone and the decode call raises TimeoutError; with the limit restored the sequence decodes on as a twin that
    never failed.
No test here faults, traps or hangs a GPU: each wait ends by its own limit."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6)
ERR_TIMEOUT = 1 << 0


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _err_word():
    from agxforge_b200 import _native as N
    w = C.c_uint32()
    N.check(N.lib().agxc_ctx_error_word(N.context(0), C.byref(w)), "error_word")
    return w.value


def _tp_reduce(torch, flag_value, wait_us):
    from agxforge.kernels import qmv as Q
    from agxforge_b200 import _native as N
    ranks, B, d, tiles = 2, 2, 256, 4
    recv = torch.arange(ranks * B * d, dtype=torch.float32, device="cuda").reshape(ranks, B, d) / 100
    flag = torch.full((1,), flag_value, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    res16 = torch.ones((B, d), dtype=torch.float16, device="cuda")
    out = torch.full((B, d), 7.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    N.check(N.lib().agxc_tp_reduce_dev(N.context(0), N.ptr(recv), ranks, 0, N.ptr(flag), N.ptr(epoch), 1, 0, tiles,
                                       N.ptr(res16), None, N.ptr(out), None, d, B, wait_us, Q._stream(torch)),
            "tp_reduce")
    torch.cuda.synchronize()
    return recv, res16, out


def test_tp_reduce_wait_for_an_unset_flag_runs_out(torch):
    _err_word()                               # clear what an earlier call left
    recv, res16, out = _tp_reduce(torch, 0, 20000)          # nobody signals: a 20 ms bound
    assert _err_word() & ERR_TIMEOUT
    assert torch.all(out == 7.0)                            # the gave-up wait wrote nothing
    # the context still works: the next kernels run and are right
    recv, res16, out = _tp_reduce(torch, 2 * 4 * 2, 2000000)  # ranks x tiles x ranks arrivals: the one-shot target
    assert _err_word() == 0
    want = recv.sum(0) + res16.float()
    assert torch.equal(out, want)


def test_fused_step_wait_limit_zero_leaves_cleanly(torch):
    from agxforge.inference import assemble
    mk = lambda: assemble.build(dict(model=dict(SMALL), bits=4, cap=64, seed=3, keep_logits=True))  # noqa: E731
    m, twin = mk(), mk()
    for x in (m, twin):
        x.set_option("fused", 1)
    assert m.fused and twin.fused
    for x in (m, twin):
        x.start(0, [4, 5, 6])
        x.decode(2, want_tokens=False)
    m.set_option("device_wait_us", 0)
    with pytest.raises(TimeoutError):
        m.decode(1, want_tokens=False)
    m.set_option("device_wait_us", 2000000)
    a_t, a_l, _ = m.decode(6, want_tokens=True, want_logits=True)
    b_t, b_l, _ = twin.decode(6, want_tokens=True, want_logits=True)
    assert np.abs(a_l - b_l).max() < 1e-3      # the failed step was undone: the same positions, the same state
    assert m.state(0)[0] == twin.state(0)[0]
    m.close()
    twin.close()
