"""Model-level parity on the B200: the whole decode step (5 kernels a layer + the head) under teacher forcing,
every step's logits against the FP64 oracle (bound 0.05 + 0.003*|ref|) and the argmax against the half-transport
oracle; the device token log, q0 and KV cache rows against the oracle's.

Small shapes run all layers; the BASELINE shapes run at full width and full vocabulary with fewer layers (the
kernels are the same per layer; depth only repeats them), so the FP64 oracle finishes in seconds."""
import numpy as np
import pytest

from oracle import decoder as D

from tests import modelcheck as MC

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _build(shape, bits=4, batch=1, cap=256, seed=0, sdt="fp16"):
    from agxforge.inference import assemble
    return assemble.build(dict(model=shape, bits=bits, batch=batch, cap=cap, seed=seed, keep_logits=True,
                               scale_dtype=sdt), keep_packs=True)


SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6)


@pytest.mark.parametrize("bits", [4, 8])
def test_small_model_forced_decode(torch, bits):
    m = _build(dict(SMALL), bits=bits)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 1024, 20).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 8, seed=2)
    MC.compare(m, seqs, lg, 8)


def test_small_model_state_and_cache(torch):
    m = _build(dict(SMALL, QKV_BIAS=True), bits=4)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, 1024, 12).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 4, seed=4)
    q0, log = m.state(0)
    T = len(seqs[0])
    assert q0 == T - 1
    assert list(log[:T]) == seqs[0]
    assert np.all(log[T:] == 0xFFFFFFFF)
    # the KV cache rows the device appended equal the half-transport oracle's rotated k and v (fp16), within 1 ulp
    om = MC.oracle_model(m)
    _, kept = om.forward(seqs[0][:T - 1], "half", keep=True)
    for l in range(m.shape.LAYERS):
        k, v = m.read_kv(l, 0, T - 1)
        kr, vr = kept[l]
        kr = kr.transpose(1, 0, 2)
        vr = vr.transpose(1, 0, 2)
        ulp_k = np.spacing(np.abs(kr).astype(np.float16)).astype(np.float64)
        ulp_v = np.spacing(np.abs(vr).astype(np.float16)).astype(np.float64)
        # later layers see inputs that already differ by rounding: allow a few ulps plus a relative slack
        assert np.all(np.abs(k.astype(np.float64) - kr) <= 8 * ulp_k + 1e-2 * np.abs(kr).max())
        assert np.all(np.abs(v.astype(np.float64) - vr) <= 8 * ulp_v + 1e-2 * np.abs(vr).max())


def test_free_generation_argmax_is_device_argmax(torch):
    """Free generation (no forcing): every token the device chose is the first argmax of the logits it produced
    (bit-exact: the same fp32 values), and the log records it."""
    m = _build(dict(SMALL), bits=4)
    m.start(0, [5, 17, 33])
    m.decode(2, want_tokens=False)
    toks, lg, _ = m.decode(6, want_tokens=True, want_logits=True)
    for i in range(6):
        assert int(toks[i, 0]) == int(np.argmax(lg[i, 0]))
    q0, log = m.state(0)
    assert q0 == 8
    assert list(log[3:9]) == [int(t) for t in toks[:, 0]]


def test_decode_host_loops_agree(torch):
    """The three host loops of agxc_decode (wait once at the end, wait for every step, one step queued ahead) run the
    same graph: the same prompts give the same free-run tokens, with and without forced inputs; other modes are
    refused."""
    outs = []
    for mode in (0, 1, 2):
        m = _build(dict(SMALL), bits=4, batch=2, seed=3)
        m.start(0, [5, 17, 33])
        m.start(1, [9, 2])
        m.decode(2, want_tokens=False)
        free, _, _ = m.decode(7, want_tokens=True, sync_each=mode)
        unset = np.full((4, 2), 0xFFFFFFFF, np.uint64)
        unset[1, 0] = 77                                   # one forced token in the middle
        forced, _, _ = m.decode(4, forced=unset, want_tokens=True, sync_each=mode)
        outs.append((free, forced, m.state(0)[0]))
        if mode == 2:
            with pytest.raises(ValueError):
                m.decode(1, sync_each=3)
        m.close()
    for free, forced, q0 in outs[1:]:
        assert np.array_equal(free, outs[0][0]) and np.array_equal(forced, outs[0][1]) and q0 == outs[0][2]


def test_batched_sequences_independent(torch):
    m = _build(dict(SMALL), bits=4, batch=3)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 1024, n).tolist() for n in (7, 15, 11)]
    seqs, lg, toks = MC.run_forced(m, prompts, 5, seed=6)
    MC.compare(m, seqs, lg, 5)


def test_qwen25_shape_two_layers(torch):
    from agxforge.inference import models
    shape = models.QWEN25_05B.replace(LAYERS=2)
    m = _build(shape, bits=4, cap=256, seed=0)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, shape.VOCAB, 40).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 4, seed=1)
    MC.compare(m, seqs, lg, 4)


def test_internlm_shape_two_layers_long_context(torch):
    from agxforge.inference import models
    shape = models.INTERNLM25_18B.replace(LAYERS=2)
    m = _build(shape, bits=4, cap=2048, seed=2)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, shape.VOCAB, 300).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 3, seed=3)
    MC.compare(m, seqs, lg, 3)


def test_internlm_q8_two_layers(torch):
    from agxforge.inference import models
    shape = models.INTERNLM25_18B.replace(LAYERS=2)
    m = _build(shape, bits=8, cap=512, seed=3)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, shape.VOCAB, 64).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 3, seed=5)
    MC.compare(m, seqs, lg, 3)


@pytest.mark.parametrize("fused", [0, 1])
def test_execute_report_keys(torch, fused):
    from agxforge.inference import execute
    m = _build(dict(SMALL), bits=4)
    m.set_option("fused", fused)
    m.start(0, [1, 2, 3])
    rep = execute.decode(m, 5, env={})  # no AGXC_* options from the environment
    for key in ("out_ids", "tokens_per_s", "per_token_ms", "gpu_ms_per_token", "host_ms_per_token",
                "dispatches_per_token", "batch"):
        assert key in rep
    assert len(rep["out_ids"]) == 5
    assert rep["dispatches_per_token"] == (1 if fused else 5 * 2 + 1)


def test_launch_trace(torch):
    """AGXC_OPT_TRACE: one step's launches in step order, each CTA entry <= its wait <= its exit, the step's kernels
    ordered by their dependency waits (no CTA passes its wait before every CTA of the predecessor reached its exit),
    and the
    traced step's tokens equal to an untraced twin's."""
    m = _build(dict(SMALL), bits=4)
    twin = _build(dict(SMALL), bits=4)
    for x in (m, twin):
        x.set_option("fused", 0)
        x.start(0, [5, 6, 7])
    m.set_option("trace", 1)
    a = m.decode(3)[0]
    tr = m.trace()
    b = twin.decode(3)[0]
    assert np.array_equal(a, b)
    assert [t["kind"] for t in tr] == ["qkv", "attn", "wo", "ffn", "down"] * 2 + ["head"]
    for t in tr:
        assert t["entry"][0] <= t["entry"][1] and t["wait"][0] <= t["wait"][1] and t["exit"][0] <= t["exit"][1]
        assert t["entry"][0] <= t["wait"][0] <= t["exit"][1]
    m.decode(1)
    one = m.trace()
    for prev, cur in zip(one, one[1:]):
        assert cur["wait"][0] >= prev["exit"][1]
    m.set_option("trace", 0)
    with pytest.raises(ValueError):
        m.trace()


def test_pdl_modes_agree(torch):
    """Programmatic dependent launch only moves when a kernel may start: plain stream order (0), the successor let in
    right after the dependency wait (1), after the inputs are staged (2) or after the last weight chunk (3) give
    bit-identical tokens and logits."""
    out = []
    for mode in (0, 1, 2, 3):
        m = _build(dict(SMALL), bits=4, seed=4)
        m.set_option("fused", 0)
        m.set_option("pdl", mode)
        m.start(0, [9, 8, 7, 6])
        toks, lg, _ = m.decode(6, want_logits=True)
        out.append((toks, lg))
        m.close()
    for toks, lg in out[1:]:
        assert np.array_equal(toks, out[0][0])
        assert np.array_equal(lg, out[0][1])


@pytest.mark.parametrize("shape,bits,layers,prompt_len", [("small", 4, 2, 20), ("small", 8, 2, 20),
                                                          ("internlm2.5-1.8b", 4, 2, 300), ("qwen2.5-0.5b", 4, 2, 40),
                                                          ("internlm2.5-1.8b", 8, 2, 70)])
def test_fused_step_against_oracle_and_kernel_path(torch, shape, bits, layers, prompt_len):
    """The batch-1 step as the fused persistent kernel and as one kernel per projection: both within the FP64 bound
    of the oracle at every step, with the argmax rule, over the same teacher-forced sequence."""
    from agxforge.inference import models
    sh = dict(SMALL) if shape == "small" else models.get(shape).replace(LAYERS=layers)
    vocab = sh["VOCAB"] if shape == "small" else sh.VOCAB
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, vocab, prompt_len).tolist()
    logits = {}
    for fused in (1, 0):
        m = _build(dict(sh) if shape == "small" else sh, bits=bits, cap=prompt_len + 16, seed=3)
        m.set_option("fused", fused)
        assert m.plan_info()["fused"]["on"] == fused
        seqs, lg, tk = MC.run_forced(m, [prompt], 6, seed=5)
        MC.compare(m, seqs, lg, 6, name="%s q%d fused=%d" % (shape, bits, fused))
        logits[fused] = lg
        m.close()
    # the two paths sum in different orders: within the GEMV bound of each other, far inside the oracle bound
    assert np.abs(logits[1] - logits[0]).max() < 1e-2


def test_fused_step_steps_back_to_back_and_free_run(torch):
    """Many fused steps in one call (the counters and accumulators alternate between two sets by the step's parity):
    free generation picks the first maximum of the device logits every step, and the token log and q0 follow."""
    m = _build(dict(SMALL), bits=4, cap=128)
    m.set_option("fused", 1)
    assert m.fused
    m.start(0, [3, 1, 4, 1, 5])
    m.decode(4, want_tokens=False)
    toks, lg, _ = m.decode(40, want_tokens=True, want_logits=True)
    for i in range(40):
        assert int(toks[i, 0]) == int(np.argmax(lg[i, 0]))
    q0, log = m.state(0)
    assert q0 == 44 and list(log[5:45]) == [int(t) for t in toks[:, 0]]
    m.close()


def test_fused_step_trace(torch):
    """The fused step's per-CTA trace: every CTA passes the qkv and FFN phases of every layer and the head, each CTA's
    phase marks (0 = a phase it had no work in) run forward in time, and no CTA met layer l + 1's qkv dependency before
    the first CTA met layer l's FFN dependency (the counters order the layers)."""
    from agxforge.inference.assemble import FUSED_TRACE_MARKS as NM
    m = _build(dict(SMALL), bits=4, cap=64)
    m.set_option("fused", 1)
    m.start(0, [5, 6, 7])
    m.set_option("trace", 1)
    m.decode(2, want_tokens=False)
    tr = m.trace_fused().astype(np.int64)
    L = m.shape.LAYERS
    assert tr.shape[0] == NM * L + 2
    for l in range(L):
        b = NM * l
        for k in (0, 1, 6, 7):
            assert np.all(tr[b + k] > 0)
        if l + 1 < L:
            assert tr[b + NM].min() >= tr[b + 6].min()
    assert np.all(tr[NM * L] > 0) and np.all(tr[NM * L + 1] > 0)
    phase_rows = [NM * l + k for l in range(L) for k in range(8)] + [NM * L, NM * L + 1]
    for c in range(tr.shape[1]):
        col = tr[phase_rows, c]
        seq = col[col > 0]
        assert np.all(np.diff(seq) >= 0)
    m.set_option("trace", 0)
    m.close()
