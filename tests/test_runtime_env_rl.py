"""Runtime env presets and RL advantage estimators (CPU)."""
import numpy as np
import pytest
import torch

from flare_b200.runtime.env import distributed_env, fault_test_env, runtime_env
from flare_b200.training.rl import compute_discounted_returns, compute_gae


def test_env_preset_merge_and_conflicts():
    env = distributed_env({"FOO": "1"})
    assert env["FOO"] == "1" and env["NCCL_NVLS_ENABLE"] == "1"
    assert fault_test_env()["NCCL_NVLS_ENABLE"] == "0"
    assert distributed_env({"NCCL_NVLS_ENABLE": "1"})["NCCL_NVLS_ENABLE"] == "1"
    with pytest.raises(ValueError):
        distributed_env({"NCCL_NVLS_ENABLE": "0"})
    assert distributed_env({"NCCL_NVLS_ENABLE": "0"}, overrides={"NCCL_NVLS_ENABLE": "0"})["NCCL_NVLS_ENABLE"] == "0"
    rt = runtime_env(peer_timeout_s=5)["env_vars"]
    assert rt["FLARE_PEER_TIMEOUT_S"] == "5" and rt["PYTHONPATH"]


def _gae_loop(r, v, d, nv, g, lam):
    adv = np.zeros(len(r))
    last = 0.0
    for t in reversed(range(len(r))):
        nxt = nv if t == len(r) - 1 else v[t + 1]
        delta = r[t] + g * nxt * (1 - d[t]) - v[t]
        last = delta + g * lam * (1 - d[t]) * last
        adv[t] = last
    return adv, adv + v


def test_gae_and_returns_match_loops():
    rng = np.random.default_rng(0)
    T, N = 17, 5
    r, v = rng.normal(size=(T, N)).astype(np.float32), rng.normal(size=(T, N)).astype(np.float32)
    d = (rng.random((T, N)) < 0.2).astype(np.float32)
    nv = rng.normal(size=N).astype(np.float32)
    adv, ret = compute_gae(torch.from_numpy(r), torch.from_numpy(v), torch.from_numpy(d), torch.from_numpy(nv),
                           0.97, 0.9)
    for n in range(N):
        a, b = _gae_loop(r[:, n], v[:, n], d[:, n], nv[n], 0.97, 0.9)
        np.testing.assert_allclose(adv[:, n].numpy(), a, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(ret[:, n].numpy(), b, rtol=1e-5, atol=1e-5)
    a1, _ = compute_gae(r[:, 0], v[:, 0], d[:, 0], float(nv[0]), 0.97, 0.9)
    assert isinstance(a1, np.ndarray)
    np.testing.assert_allclose(a1, adv[:, 0].numpy(), rtol=1e-6)
    rets = compute_discounted_returns(r[:, 1], d[:, 1], 0.9)
    run, want = 0.0, np.zeros(T)
    for t in reversed(range(T)):
        if d[t, 1]:
            run = 0.0
        run = r[t, 1] + 0.9 * run
        want[t] = run
    np.testing.assert_allclose(rets, want, rtol=1e-5, atol=1e-6)


def _exp(r, v=0.0, d=0.0):
    from flare_b200.training.rl import Experience

    return Experience({"x": r}, 0, r, {"x": r}, d, values=v)


def test_replay_buffer_ring_and_prioritized_sampling():
    import numpy as np

    from flare_b200.training.rl import ReplayBuffer, ReplayBufferSpec

    buf = ReplayBuffer(ReplayBufferSpec(capacity=4, batch_size=2))
    for i in range(6):
        buf.push(_exp(float(i)))
    assert buf.size() == 4 and sorted(e.rewards for e in buf.items) == [2.0, 3.0, 4.0, 5.0]  # oldest overwritten
    pb = ReplayBuffer(ReplayBufferSpec(capacity=8, batch_size=4000, prioritized=True, alpha=1.0, beta=1.0), seed=1)
    for i in range(4):
        pb.push(_exp(float(i)))
    pb.update_priorities([0, 1, 2, 3], [1.0, 1.0, 1.0, 7.0])
    ex, idx, w = pb.sample()
    assert abs(np.mean(idx == 3) - 0.7) < 0.03  # P(3) = 7 / 10
    assert abs(w[idx == 3][0] - 1.0 / 7.0) < 1e-6 and w.max() == 1.0  # (N P)^-beta / max (priorities + eps)


def test_rollout_buffer_gae_matches_compute_gae():
    import torch

    from flare_b200.training.rl import RolloutBuffer, RolloutBufferSpec, compute_gae

    rb = RolloutBuffer(RolloutBufferSpec(buffer_size=5, gamma=0.9, gae_lambda=0.8))
    rs, vs, ds = [1.0, 0.0, 2.0, -1.0, 0.5], [0.2, 0.1, 0.4, 0.0, 0.3], [0.0, 0.0, 1.0, 0.0, 0.0]
    for r, v, d in zip(rs, vs, ds):
        rb.push(_exp(r, v, d))
    adv, ret = rb.finish(next_value=0.25)
    a2, r2 = compute_gae(torch.tensor(rs), torch.tensor(vs), torch.tensor(ds), 0.25, 0.9, 0.8)
    torch.testing.assert_close(adv, a2)
    torch.testing.assert_close(ret, r2)
    ex, a, r = rb.sample(3)
    assert len(ex) == 3 and a.shape == (3,)
