"""The asynchronous chunk scheduler on a CUDA policy (inference enqueued on
its own stream, results copied to pinned host memory behind an event) gives
the same actions as synchronous predict_action_chunk calls with the same
states and noise; PrefillDecodeStreams orders a decode after its prefill."""
import numpy as np
import pytest
import torch

from reflex_b200.config import pi05_config

from test_gpu_policy import _model_with_cached_prefix

pytestmark = pytest.mark.gpu


class FixedNoise:
    def __init__(self, pol, noise):
        self.pol, self.noise = pol, noise

    def predict_action_chunk(self, batch, **kw):
        return self.pol.predict_action_chunk(batch, noise=self.noise, **kw)


def test_async_schedule_matches_synchronous_chunks():
    from reflex_b200.policy import PI0Model, PI0Policy
    from reflex_b200.config import pi0_config
    from reflex_b200.scheduler import ChunkScheduler
    cfg = pi0_config(num_layers=2, quant_mode="u8_ref", chunk_size=8)
    m, wts, ctx, x0, st = _model_with_cached_prefix(cfg, 64, PI0Model)
    pol = PI0Policy(m, n_action_steps=6)
    noise = x0.cuda()
    sch = ChunkScheduler(FixedNoise(pol, noise), 6, 2)
    obs = {"observation.state": st.cuda()}
    acts = [sch.get_action(obs) for _ in range(12)]
    sch.wait()  # the third chunk, launched at step 10, still owns the engine
    # the same two chunks synchronously: the first from the observed state,
    # the second from the first chunk's last executed action as the state
    c1 = pol.predict_action_chunk(obs, noise=noise)[0].cpu().numpy()
    s2 = torch.zeros_like(st)
    s2[0, :cfg.action_dim] = torch.from_numpy(c1[5, :cfg.state_dim])
    c2 = pol.predict_action_chunk({"observation.state": s2.cuda()}, noise=noise)[0].cpu().numpy()
    for i in range(6):
        assert np.array_equal(acts[i], c1[i])
        assert np.array_equal(acts[6 + i], c2[i])


def test_prefill_then_decode_streams():
    from reflex_b200.scheduler import PrefillDecodeStreams
    ex = PrefillDecodeStreams()
    src = torch.arange(1 << 20, dtype=torch.float32, device="cuda")
    dst = torch.zeros_like(src)

    def prefill():
        torch.cuda._sleep(20_000_000)  # a long prefill: the decode must still see its result
        dst.copy_(src)

    ex.concurrent_prefill(prefill)
    out = ex.concurrent_decode(lambda: dst.sum())
    ex.synchronize_streams()
    assert out.item() == src.sum().item()
