"""Host logic of the asynchronous chunk scheduler (reflex_b200.scheduler)
against the reference's control loop (reflex/run.py:47-252,
run_streaming.py:104-175): chunk bootstrap, launch point overlap_steps
before the chunk end, future-state substitution (the last action of the
executing chunk, zero-padded or truncated to the state width), chunk switch,
and incremental_input in streaming mode.  CPU policy, no GPU."""
import numpy as np
import pytest

from reflex_b200.scheduler import ChunkScheduler


class FakePolicy:
    def __init__(self, n, a):
        self.n, self.a, self.calls = n, a, []

    def predict_action_chunk(self, batch, **kw):
        self.calls.append((np.array(batch["observation.state"]), kw))
        k = len(self.calls)
        return (np.arange(self.n * self.a, dtype=np.float32).reshape(1, self.n, self.a) + 1000 * k)


@pytest.mark.parametrize("state_dim,action_dim", [(8, 7), (6, 7)])
def test_schedule_and_future_state(state_dim, action_dim):
    n, overlap = 5, 2
    pol = FakePolicy(n, action_dim)
    sch = ChunkScheduler(pol, n, overlap)
    obs = {"observation.state": np.full(state_dim, -1.0, dtype=np.float32)}
    acts = [sch.get_action(obs) for _ in range(3 * n)]
    chunks = [np.arange(n * action_dim, dtype=np.float32).reshape(n, action_dim) + 1000 * k for k in (1, 2, 3, 4)]
    for step, a in enumerate(acts):
        assert np.array_equal(a, chunks[step // n][step % n]), step
    # inferences: the bootstrap at step 0, then at index n - overlap of every chunk
    assert [l["chunk_index"] for l in sch.launches] == [0, n - overlap, n - overlap, n - overlap]
    assert np.array_equal(pol.calls[0][0], obs["observation.state"])
    for k in (1, 2, 3):
        last = chunks[k - 1][n - 1]
        want = np.zeros(state_dim, dtype=np.float32)
        m = min(state_dim, action_dim)
        want[:m] = last[:m]
        assert np.array_equal(pol.calls[k][0], want)


def test_streaming_passes_incremental_input_after_the_first_chunk():
    pol = FakePolicy(4, 3)
    sch = ChunkScheduler(pol, 4, 1, streaming=True)
    obs = {"observation.state": np.zeros(3, dtype=np.float32)}
    for _ in range(9):
        sch.get_action(obs)
    assert [c[1]["incremental_input"] for c in pol.calls] == [False, True, True]


def test_argument_checks():
    with pytest.raises(ValueError):
        ChunkScheduler(FakePolicy(4, 3), 4, 5)
    with pytest.raises(ValueError):
        ChunkScheduler(FakePolicy(4, 3), 4, -1)
    sch = ChunkScheduler(FakePolicy(4, 3), 4, 0)
    assert sch.should_fetch_observation() and not sch.is_running()
    with pytest.raises(RuntimeError):
        sch.get_current_action()


def test_wait_returns_with_or_without_a_pending_inference():
    pol = FakePolicy(4, 3)
    sch = ChunkScheduler(pol, 4, 2)
    sch.wait()  # nothing pending
    obs = {"observation.state": np.zeros(3, dtype=np.float32)}
    for _ in range(3):  # the second inference is launched at index 2 (host policy: completed at once)
        sch.get_action(obs)
    assert sch.next_chunk is not None
    sch.wait()
