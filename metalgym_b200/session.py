"""Python mirror of the drop-in C++ API (include/metalgym/gym.h, ppo.h) over
the mg_gym_* / mg_ppo_* C ABI: the same method and field names as the
reference's Gym<Env> (gym.h:15-121) and PPOModel<Env> (model/ppo.h:106-1009),
with device buffers read back as numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import check, lib

GYM_BUF = dict(states=0, actions=1, obs=2, reward=3, done=4, rng=5)
PPO_BUF = dict(obs=0, actions=1, logp=2, value=3, reward=4, done=5, adv=6, ret=7, head=8, weights=9, master=10,
               momentum=11, variance=12, grad=13, stats=14, adv_stats=15, train_head=16)


class Gym:
    """Gym<Env>(parallels): the env buffers of one device (gym.h:36-72)."""

    def __init__(self, kernel_name: str, parallels: int, seed: int = 0, first_env_id: int = 0, device: int = -1):
        self._h = C.c_void_p()
        check(lib().mg_gym_create(kernel_name.encode(), parallels, seed, first_env_id, device, C.byref(self._h)),
              "mg_gym_create")
        info = (C.c_uint32 * 8)()
        check(lib().mg_gym_info(self._h, info))
        (self.parallels, self.state_bytes, self.action_bytes, self.obs_bytes, self.obs_dim, self.act_dim,
         cont, self.device) = list(info)
        self.continuous = bool(cont)
        self.kernel_name = kernel_name

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            # a model borrows its gym (model/ppo.h:145-147): close the models first
            for m in list(getattr(self, "_models", ())):
                m.close()
            lib().mg_gym_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def action_dtype(self):
        return np.float32 if self.continuous else np.int32

    def run(self, actions: np.ndarray | None, reward_out: np.ndarray | None = None) -> np.ndarray:
        """gym.run (gym.h:110-121): one step with host actions, rewards back."""
        n = self.parallels
        if reward_out is None:
            reward_out = np.zeros(n, np.float32)
        a = None if actions is None else np.ascontiguousarray(actions, dtype=self.action_dtype())
        check(lib().mg_gym_run(self._h, None if a is None else a.ctypes.data, reward_out.ctypes.data,
                               len(reward_out)), "mg_gym_run")
        return reward_out

    def run_random(self, steps: int, mode: int = 0) -> None:
        check(lib().mg_gym_run_random(self._h, steps, mode), "mg_gym_run_random")

    def synchronize(self):
        check(lib().mg_gym_synchronize(self._h))

    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().mg_gym_stream(self._h, C.byref(s)))
        return s.value or 0

    def buffer(self, which: str):
        p, n = C.c_void_p(), C.c_size_t()
        check(lib().mg_gym_buffer(self._h, GYM_BUF[which], C.byref(p), C.byref(n)))
        return p.value, n.value

    def download(self, which: str) -> np.ndarray:
        _, n = self.buffer(which)
        out = np.zeros(n, np.uint8)
        check(lib().mg_gym_download(self._h, GYM_BUF[which], out.ctypes.data, n))
        return out

    def upload(self, which: str, data: np.ndarray) -> None:
        d = np.ascontiguousarray(data)
        check(lib().mg_gym_upload(self._h, GYM_BUF[which], d.ctypes.data, d.nbytes))

    def obs(self) -> np.ndarray:
        return self.download("obs").view(np.float32).reshape(self.parallels, self.obs_dim)

    def done(self) -> np.ndarray:
        return self.download("done")


class PPOModel:
    """PPOModel<Env>(gym, e, s, layers, lr, T, seed) (model/ppo.h:274-446)."""

    def __init__(self, gym: Gym, embed: int, scale: int, layers: int, lr: float, horizon: int = 32, seed: int = 0):
        self.gym = gym
        self._h = C.c_void_p()
        if not hasattr(gym, "_models"):
            gym._models = weakref.WeakSet()
        gym._models.add(self)
        check(lib().mg_ppo_create(gym.handle, embed, scale, layers, lr, horizon, seed, C.byref(self._h)),
              "mg_ppo_create")
        info = (C.c_uint64 * 12)()
        check(lib().mg_ppo_info(self._h, info))
        (self.rows, self.obs_dim, self.act_dim, self.embed, self.hidden, self.layers, self.horizon, self.opt_count,
         self.opt_float_count, self.param_count, cont, self.action_bytes) = [int(x) for x in info]
        self.continuous = bool(cont)

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().mg_ppo_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- hyperparameters (model/ppo.h:186-191)
    def hyper(self) -> dict:
        v = (C.c_float * 6)()
        check(lib().mg_ppo_get_hyper(self._h, v))
        return dict(zip(("clip", "valueCoef", "entropyCoef", "maxGradNorm", "gamma", "lambda"), list(v)))

    def set_hyper(self, **kw) -> None:
        h = self.hyper()
        h.update(kw)
        check(lib().mg_ppo_set_hyper(self._h, h["clip"], h["valueCoef"], h["entropyCoef"], h["maxGradNorm"],
                                     h["gamma"], h["lambda"]))

    # ---- the hot path
    def collect(self):
        check(lib().mg_ppo_collect(self._h), "collect")

    def train(self, epochs: int = 4):
        check(lib().mg_ppo_train(self._h, epochs), "train")

    def train_slot(self, t: int):
        check(lib().mg_ppo_train_slot(self._h, t), "trainSlot")

    def p2p_handle(self) -> bytes:
        """This rank's 64-byte exchange-region handle (mg_ppo_p2p_handle)."""
        buf = (C.c_char * 64)()
        check(lib().mg_ppo_p2p_handle(self._h, buf), "p2p_handle")
        return bytes(buf)

    def p2p_open(self, handles: list, rank: int, world: int) -> None:
        """Opens every rank's region (handles in rank order; mg_ppo_p2p_open)."""
        blob = b"".join(handles)
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        check(lib().mg_ppo_p2p_open(self._h, buf, rank, world), "p2p_open")

    def save(self, path) -> None:
        """Checkpoint of the training state (mg_ppo_save)."""
        check(lib().mg_ppo_save(self._h, str(path).encode()), "save")

    def load(self, path) -> None:
        """Restores a checkpoint of a model of the same shapes (mg_ppo_load)."""
        check(lib().mg_ppo_load(self._h, str(path).encode()), "load")

    @property
    def minibatch_rows(self) -> int:
        """Rows per training minibatch: 0 = one time slot (the reference)."""
        v = C.c_int()
        check(lib().mg_ppo_minibatch_rows(self._h, C.byref(v)))
        return v.value

    @minibatch_rows.setter
    def minibatch_rows(self, rows: int):
        check(lib().mg_ppo_set_minibatch_rows(self._h, int(rows)), "minibatchRows")

    @property
    def collect_fused(self) -> bool:
        """Whether the next collect() runs as one persistent kernel
        (mg_ppo_collect_fused). Set True / False to choose the kernel / the
        per-step graph, None for the library's choice (the default: the kernel
        where it applies, up to 4096 parallels)."""
        v = C.c_int()
        check(lib().mg_ppo_collect_fused(self._h, C.byref(v)))
        return bool(v.value)

    @collect_fused.setter
    def collect_fused(self, on):
        mode = -1 if on is None else (1 if on else 0)
        check(lib().mg_ppo_set_collect_fused(self._h, mode), "collect_fused")

    @property
    def fused_minibatch(self) -> bool:
        """A minibatch's block forwards, head and block backwards as one kernel
        where they apply (mg_ppo_set_fused_minibatch; off by default)."""
        v = C.c_int()
        check(lib().mg_ppo_fused_minibatch(self._h, C.byref(v)))
        return bool(v.value)

    @fused_minibatch.setter
    def fused_minibatch(self, on: bool):
        check(lib().mg_ppo_set_fused_minibatch(self._h, 1 if on else 0), "fused_minibatch")

    def train_rows(self, key, base: int):
        """One row-mode minibatch over rows perm(base .. base + B - 1) of the
        permutation keyed by the four words of key."""
        k = (C.c_uint32 * 4)(*[int(x) & 0xFFFFFFFF for x in key])
        check(lib().mg_ppo_train_rows(self._h, k, int(base)), "trainRows")

    def forward(self):
        check(lib().mg_ppo_forward(self._h), "forward")

    def last_stats(self) -> dict:
        v = (C.c_float * 6)()
        check(lib().mg_ppo_last_stats(self._h, v))
        return dict(zip(("policy", "value", "entropy", "approxKl", "clipFrac", "gradNorm"), list(v)))

    def set_log_std(self, v: float):
        check(lib().mg_ppo_set_log_std(self._h, v))

    def log_std_value(self, k: int) -> float:
        f = C.c_float()
        check(lib().mg_ppo_log_std(self._h, k, C.byref(f)))
        return f.value

    def step_counter(self) -> float:
        f = C.c_float()
        check(lib().mg_ppo_step_counter(self._h, C.byref(f)))
        return f.value

    def set_step_counter(self, v: float):
        check(lib().mg_ppo_set_step_counter(self._h, v))

    def phase_ms(self) -> tuple[float, float]:
        """Device time (ms) of the last collect() and train() (mg_ppo_phase_ms)."""
        v = (C.c_float * 2)()
        check(lib().mg_ppo_phase_ms(self._h, v))
        return float(v[0]), float(v[1])

    def graph_kernels(self) -> tuple[int, int]:
        """Kernel launches per replay of the collect and train graphs."""
        v = (C.c_uint64 * 2)()
        check(lib().mg_ppo_graph_kernels(self._h, v))
        return int(v[0]), int(v[1])

    def set_allreduce_overlap(self, on: bool):
        """All-reduce all but the last backward layer's gradients while that
        layer's backward runs (mg_ppo_set_allreduce_overlap; NCCL, world > 1)."""
        check(lib().mg_ppo_set_allreduce_overlap(self._h, 1 if on else 0), "allreduce_overlap")

    def set_comm_timeout(self, seconds: float):
        """Failure detection of data-parallel train() (mg_ppo_set_comm_timeout):
        > 0 turns an all-reduce that fails on a peer, or does not finish in
        time, into an error (code 6) after aborting the communicator."""
        check(lib().mg_ppo_set_comm_timeout(self._h, float(seconds)), "comm_timeout")

    def set_comm(self, comm, rank: int, world: int):
        check(lib().mg_ppo_set_comm(self._h, comm, rank, world))

    # ---- buffers
    def param_info(self, i: int):
        off, cnt, gf = C.c_uint64(), C.c_uint32(), C.c_int()
        check(lib().mg_ppo_param_info(self._h, i, C.byref(off), C.byref(cnt), C.byref(gf)))
        return off.value, cnt.value, bool(gf.value)

    def buffer(self, which: str, slot: int = -1):
        p, n = C.c_void_p(), C.c_size_t()
        check(lib().mg_ppo_buffer(self._h, PPO_BUF[which], slot, C.byref(p), C.byref(n)))
        return p.value, n.value

    def download(self, which: str, slot: int = -1) -> np.ndarray:
        _, n = self.buffer(which, slot)
        out = np.zeros(n, np.uint8)
        check(lib().mg_ppo_download(self._h, PPO_BUF[which], slot, out.ctypes.data, n))
        return out

    def upload(self, which: str, data: np.ndarray, slot: int = -1) -> None:
        d = np.ascontiguousarray(data)
        check(lib().mg_ppo_upload(self._h, PPO_BUF[which], slot, d.ctypes.data, d.nbytes))

    def slots(self, which: str) -> np.ndarray:
        """All slots of a slot buffer as [T (+1 for obs)] x rows (x dim)."""
        raw = self.download(which)
        R, T = self.rows, self.horizon
        if which == "obs":
            return raw.view(np.float32).reshape(T + 1, R, self.obs_dim)
        if which == "actions":
            if self.continuous:
                return raw.view(np.float32).reshape(T, R, self.act_dim)
            return raw.view(np.int32).reshape(T, R)
        if which == "done":
            return raw.reshape(T, R)
        return raw.view(np.float32).reshape(T, R)


def minibatch_rows(key, base: int, rows: int, total: int):
    """Flat slot-major rollout rows read by rows q < rows of the row-mode
    minibatch starting at permuted position base (host evaluation of the
    same permutation the kernels use)."""
    k = (C.c_uint32 * 4)(*[int(x) & 0xFFFFFFFF for x in key])
    out = np.zeros(rows, np.uint64)
    check(lib().mg_minibatch_rows(k, int(base), int(rows), int(total), out.ctypes.data_as(C.c_void_p)),
          "mg_minibatch_rows")
    return out

