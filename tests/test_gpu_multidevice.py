"""Sessions sharded over two GPUs of one process (a context opened on devices 0 and 1): every
session's tokens must equal those of the same session on one GPU, for greedy generation, the
sampling policy, the scheduler, and prefill and appends with their logits (sessions never interact, and draws are keyed by the global
session index or the request). Skipped on a box with one GPU."""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth

pytestmark = pytest.mark.gpu


def _two_gpus():
    import torch
    return torch.cuda.device_count() >= 2


@pytest.mark.skipif("not _two_gpus()")
def test_two_devices_match_one():
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": 512})
    data = synth.build_model_file(spec)
    n, P, T = 64, 24, 10
    prompts = synth.prompts_uniform_fast(n, P, spec.vocab, seed=13)
    lens = (np.arange(n) % P + 1).astype(np.int32)
    sp = quant.Sampling(0.8, 1.2, 40, 0.9, 6, True)
    out = {}
    for devs in ((0,), (0, 1)):
        ctx = quant.Context(devs)
        m = quant.Model.decode(data, ctx)
        b = m.new_batch(n, 0, P)
        g = b.generate(prompts, lens, T)[0]
        pol = b.generate_policy(prompts, lens, T, sp, penalize_prompt=True, session0=5)[0]
        # prefill and appends with logits: each shard's outputs come back through its own staging
        lg, tok, pr = b.prefill(prompts, lens, want_logits=True)
        steps = [(lg.copy(), tok.copy(), pr.copy())]
        for _ in range(3):
            lg, tok, pr = b.append(tok, want_logits=True)
            steps.append((lg.copy(), tok.copy(), pr.copy()))
        b.close()
        sched = quant.Scheduler(m, 16, sp, max_prompt=P, max_new=T)
        ids = [sched.submit(prompts[i, :lens[i]], T - i % 4, draw_key=100 + i) for i in range(n)]
        sched.run(4)
        sc = [sched.result(r)[0].tolist() for r in ids]
        sched.close()
        m.close()
        ctx.close()
        out[devs] = (g, pol, sc, steps)
    a, b2 = out[(0,)], out[(0, 1)]
    np.testing.assert_array_equal(a[0], b2[0])
    np.testing.assert_array_equal(a[1], b2[1])
    assert a[2] == b2[2]
    for (l1, t1, p1), (l2, t2, p2) in zip(a[3], b2[3]):
        np.testing.assert_array_equal(t1, t2)
        np.testing.assert_allclose(p1, p2, rtol=1e-6)
        np.testing.assert_allclose(l1, l2, rtol=1e-5, atol=1e-6)


@pytest.mark.skipif("not _two_gpus()")
def test_entry_points_leave_the_callers_device():
    """Calls on a context spanning devices 0 and 1 switch to each shard's device and back: the
    caller's current device is the same after every call (a caller's own kernels, and the _dev
    entry points on the default stream, run on the current device)."""
    import torch
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": 512})
    data = synth.build_model_file(spec)
    n, P = 32, 16
    prompts = synth.prompts_uniform_fast(n, P, spec.vocab, seed=17)
    lens = np.full(n, P, np.int32)
    for cur in (0, 1):
        torch.cuda.set_device(cur)
        ctx = quant.Context((0, 1))
        m = quant.Model.decode(data, ctx)
        assert torch.cuda.current_device() == cur
        b = m.new_batch(n, 0, P, top_k=8)
        b.generate(prompts, lens, 4)
        assert torch.cuda.current_device() == cur
        b.generate_limits(prompts, lens, np.full(n, 3, np.int32), temperature=0.7)
        b.score(prompts, lens)
        b.prefill(prompts, lens)
        assert torch.cuda.current_device() == cur
        b.close()
        m.close()
        ctx.close()
        assert torch.cuda.current_device() == cur
    torch.cuda.set_device(0)
