"""Engine-level parity with the oracle at the shapes the benchmark runs
(BASELINE configs[1]-[4]), not only at small row counts:

* configs[1]/[2]: collect() of 4096 CartPole envs, T = 32, embed 128, hidden
  512, 2 blocks (the fused collect kernel, the default path there), replayed
  teacher-forced on the CPU (tests/test_engine.py::replay_collect): env
  steps, resets, RNG words and GAE bit-exact, values / log-probs within rel
  1e-2; then trainSlot on one whole 4096-row slot against the oracle's
  minibatch (loss statistics rel 2e-2, per-parameter gradient relative L2 <
  3e-2, Adam direction);
* a row-mode minibatch of 8192 rows drawn from the 16384 x 32
  CartPoleContinuous rollout (the Gaussian head and the learned log-std);
* a row-mode minibatch of 32768 rows drawn from the 262144 x 32
  VoxelNav rollout at embed 256, hidden 1024, 4 blocks.

The oracle is the C++ restatement of model/ppo.h (oracle/mg_oracle.cpp,
OpenMP over rows), pinned to the reference's own sources by
tests/test_oracle_pin.py and tests/test_ref_host.py."""
import numpy as np
import pytest

from orc import ptr
from test_engine import compare_minibatch, copy_optimiser_state, make, oracle_model, replay_collect

pytestmark = pytest.mark.gpu


def test_config2_collect_teacher_forced_4096(mg, oracle, hostenv):
    gym, model = make("rollout_cartpole", 4096, 128, 4, 2, 32, seed=1)
    assert model.collect_fused  # the default path at this shape
    model.collect()
    replay_collect(oracle, hostenv, model, "rollout_cartpole", 1)


@pytest.mark.parametrize("fused_minibatch", [False, True])
def test_config3_train_slot_4096_rows(mg, oracle, fused_minibatch):
    R, T = 4096, 32
    gym, model = make("rollout_cartpole", R, 128, 4, 2, T, seed=2)
    model.fused_minibatch = fused_minibatch
    model.collect()
    om = oracle_model(oracle, model, 2)
    copy_optimiser_state(oracle, om, model)
    t = 17
    cols = [np.ascontiguousarray(model.slots(k)[t]) for k in ("obs", "actions", "adv", "ret", "logp")]
    stats = np.zeros((R, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    m0 = model.download("master").view(np.float32).copy()
    oracle.orc_model_set_step_counter(om, model.step_counter())
    oracle.orc_model_train_minibatch(om, *[ptr(c) for c in cols], R, ptr(stats), ptr(nsq))
    model.train_slot(t)
    compare_minibatch(oracle, om, model, stats, nsq, m0)
    oracle.orc_model_destroy(om)


def _row_minibatch(oracle, name, R, E, L, B, seed, key, base):
    from metalgym_b200.session import minibatch_rows

    T = 32
    gym, model = make(name, R, E, 4, L, T, seed=seed)
    model.minibatch_rows = B
    model.collect()
    om = oracle_model(oracle, model, seed)
    copy_optimiser_state(oracle, om, model)
    idx = minibatch_rows(key, base, B, T * R).astype(np.int64)
    t, i = idx // R, idx % R
    assert len(np.unique(t)) == T  # the minibatch mixes every slot
    cols = [np.ascontiguousarray(model.slots(k)[t, i]) for k in ("obs", "actions", "adv", "ret", "logp")]
    stats = np.zeros((B, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    m0 = model.download("master").view(np.float32).copy()
    oracle.orc_model_set_step_counter(om, model.step_counter())
    oracle.orc_model_train_minibatch(om, *[ptr(c) for c in cols], B, ptr(stats), ptr(nsq))
    model.train_rows(key, base)
    compare_minibatch(oracle, om, model, stats, nsq, m0)
    oracle.orc_model_destroy(om)
    return model


def test_config4_row_minibatch_8192_of_16384_continuous(mg, oracle):
    model = _row_minibatch(oracle, "rollout_cartpole_continuous", 16384, 128, 2, 8192, 6,
                           [0x1234, 0x5678, 0x9ABC, 0xDEF0], 5 * 8192)
    assert np.isfinite(model.log_std_value(0))


def test_config5_row_minibatch_32768_voxelnav(mg, oracle):
    _row_minibatch(oracle, "rollout_voxelnav", 262144, 256, 4, 32768, 8, [7, 77, 777, 7777], 100 * 32768)
