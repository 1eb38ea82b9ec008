"""One training minibatch's block forwards, head and block backwards as one
kernel (metalgym_b200/csrc/minibatch_tiles.cu, mg_ppo_set_fused_minibatch)
against the separate cluster kernels it merges (k_block_cluster,
k_head_tail). The passes are the same code on the same data in the same
order, so everything must be bit-identical: the gradient arena, the Adam
state and weights after the step, the per-row loss statistics, the saved
activations and the head rows; over whole train() calls (the captured graph)
as well as single trainSlot / trainRows minibatches, for 1 and 2 blocks,
ragged tile counts and row-mode minibatches. The separate kernels are pinned
to the oracle and to torch by their own tests (test_engine.py,
test_block_cluster.py, test_head_tail.py); test_parity_full_shapes.py checks
a 4096-row minibatch of the merged kernel against the oracle as well."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STATE = ("grad", "master", "momentum", "variance", "weights")


def make(R, L, T, seed, fused):
    from metalgym_b200.session import Gym, PPOModel

    gym = Gym("rollout_cartpole", R, seed=0)
    model = PPOModel(gym, 128, 4, L, 3e-4, T, seed)
    model.fused_minibatch = fused
    return gym, model


def same(a, b, what):
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), what


@pytest.mark.parametrize("R,L", [(4096, 2), (1024, 1), (640, 2)])
def test_train_slot_bit_identical(mg, R, L):
    T = 4
    (_, sep), (_, fus) = make(R, L, T, 5, False), make(R, L, T, 5, True)
    assert fus.fused_minibatch and not sep.fused_minibatch
    for m in (sep, fus):
        m.collect()
    for t in (1, 3):
        sep.train_slot(t)
        fus.train_slot(t)
        for k in STATE + ("train_head",):
            same(sep.download(k), fus.download(k), f"slot {t}: {k}")
        assert sep.last_stats() == fus.last_stats()


@pytest.mark.parametrize("R,L", [(4096, 2), (2048, 1)])
def test_train_graph_bit_identical_and_fewer_launches(mg, R, L):
    """Two iterations of collect() + train(2) through the captured graphs:
    identical weights and Adam state, and the merged kernel replaces 2L + 1
    launches per minibatch by one."""
    T = 8
    (_, sep), (_, fus) = make(R, L, T, 7, False), make(R, L, T, 7, True)
    for it in range(2):
        for m in (sep, fus):
            m.collect()
            m.train(2)
        for k in STATE:
            same(sep.download(k), fus.download(k), f"iteration {it}: {k}")
        assert sep.last_stats() == fus.last_stats()
    k_sep, k_fus = sep.graph_kernels()[1], fus.graph_kernels()[1]
    assert k_sep - k_fus == 2 * L * T, (k_sep, k_fus)


def test_row_mode_minibatches_bit_identical(mg):
    """Row-subset minibatches (the row permutation gathers the observations,
    actions and advantages of every row) through both paths."""
    R, T = 2048, 4
    (_, sep), (_, fus) = make(R, 2, T, 9, False), make(R, 2, T, 9, True)
    for m in (sep, fus):
        m.minibatch_rows = 4096
        m.collect()
    for base in (0, 4096):
        sep.train_rows([11, 22, 33, 44], base)
        fus.train_rows([11, 22, 33, 44], base)
        for k in STATE:
            same(sep.download(k), fus.download(k), f"rows from {base}: {k}")
    for m in (sep, fus):
        m.collect()
        m.train(1)
    for k in STATE:
        same(sep.download(k), fus.download(k), f"train(1): {k}")


def test_switch_recaptures_the_train_graph(mg):
    """Turning the merged kernel off and on between train() calls recaptures
    the graph and continues the same training."""
    R, T = 1024, 4
    (_, ref), (_, mixed) = make(R, 2, T, 3, True), make(R, 2, T, 3, True)
    for on in (False, True, False):
        mixed.fused_minibatch = on
        for m in (ref, mixed):
            m.collect()
            m.train(1)
        same(ref.download("master"), mixed.download("master"), f"fused_minibatch={on}")
