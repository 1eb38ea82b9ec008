"""Environment authoring (include/metalgym/register_env.cuh), CPU only.

A user environment is a struct with __host__ __device__ reset / step, moved
from its Metal source, and one MG_REGISTER_ENV line. Its translation unit is
compiled for sm_100a against the public headers alone (no library sources)
and loaded next to the product library; loading registers its kernels under
Env::KERNEL. Environments whose State fits in registers (at most 64 bytes)
and whose observation has at most 32 floats also register the persistent
collect() kernel (mg_env_ops::collect_fused); larger ones register NULL there
and keep the per-step collect graph. nvcc cross-compiles without a GPU, and
registration makes no CUDA call, so this runs on the CPU.
"""
import ctypes
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB_DIR = ROOT / "metalgym_b200"
NVCC = "/usr/local/cuda/bin/nvcc"

USER_ENV = r"""
#include "metalgym/register_env.cuh"

// A one-dimensional walk: three actions move the walker left, not at all or
// right; the episode ends after 50 steps or 2 units from the start.
struct Walk {
    struct State { float x; uint32_t t; };
    using Action = int;
    struct Obs { float x; float t; };
    static constexpr uint32_t OBS_DIM = 2;
    static constexpr uint32_t ACT_DIM = 3;
    static constexpr const char* KERNEL = "rollout_test_walk";
    __host__ __device__ static void reset(State& s, uint32_t& rng) {
        s.x = rngUniform(rng, -0.5f, 0.5f);
        s.t = 0;
    }
    __host__ __device__ static void step(State& s, Action a, Obs& o, float& reward, uint8_t& done) {
        s.x += 0.1f * (float)(a - 1);
        s.t += 1;
        o.x = s.x;
        o.t = (float)s.t;
        reward = -fabsf(s.x);
        done = (s.t >= 50 || fabsf(s.x) > 2.0f) ? 1 : 0;
    }
};

// The same walk with a 256-byte trail in its State: stepped in place in
// global memory, so no fused collect kernel.
struct TrailWalk {
    struct State { float x; uint32_t t; float trail[62]; };
    using Action = int;
    struct Obs { float x; float t; };
    static constexpr uint32_t OBS_DIM = 2;
    static constexpr uint32_t ACT_DIM = 3;
    static constexpr const char* KERNEL = "rollout_test_trail_walk";
    __host__ __device__ static void reset(State& s, uint32_t& rng) {
        s.x = rngUniform(rng, -0.5f, 0.5f);
        s.t = 0;
    }
    __host__ __device__ static void step(State& s, Action a, Obs& o, float& reward, uint8_t& done) {
        s.trail[s.t % 62] = s.x;
        s.x += 0.1f * (float)(a - 1);
        s.t += 1;
        o.x = s.x;
        o.t = (float)s.t;
        reward = -fabsf(s.x);
        done = s.t >= 50 ? 1 : 0;
    }
};

// A continuous walk (Gaussian head): the action is a struct of ACT_DIM floats.
struct Glide {
    struct State { float x, v; uint32_t t; };
    struct Action { float push; };
    struct Obs { float x, v; };
    static constexpr uint32_t OBS_DIM = 2;
    static constexpr uint32_t ACT_DIM = 1;
    static constexpr const char* KERNEL = "rollout_test_glide";
    __host__ __device__ static void reset(State& s, uint32_t& rng) {
        s.x = rngUniform(rng, -0.5f, 0.5f);
        s.v = 0.0f;
        s.t = 0;
    }
    __host__ __device__ static void step(State& s, Action a, Obs& o, float& reward, uint8_t& done) {
        s.v += 0.05f * fminf(fmaxf(a.push, -1.0f), 1.0f);
        s.x += s.v;
        s.t += 1;
        o.x = s.x;
        o.v = s.v;
        reward = -fabsf(s.x);
        done = s.t >= 100 ? 1 : 0;
    }
};

// The eligibility limits: a State of 64 bytes and 32 observations qualify.
template <int STATE_WORDS, int OBS>
struct Sized {
    struct State { float w[STATE_WORDS]; };
    using Action = int;
    struct Obs { float o[OBS]; };
    static constexpr uint32_t OBS_DIM = OBS;
    static constexpr uint32_t ACT_DIM = 2;
    static constexpr const char* KERNEL = "rollout_test_sized";
    __host__ __device__ static void reset(State& s, uint32_t& rng) {
        for (int i = 0; i < STATE_WORDS; i++) s.w[i] = rngUniform(rng);
    }
    __host__ __device__ static void step(State& s, Action a, Obs& o, float& reward, uint8_t& done) {
        for (int i = 0; i < OBS; i++) o.o[i] = s.w[i % STATE_WORDS] + (float)a;
        reward = 0.0f;
        done = 0;
    }
};

static_assert(mg::collect_fused_eligible<Walk>(), "a 8-byte State fits in registers");
static_assert(!mg::collect_fused_eligible<TrailWalk>(), "a 256-byte State is stepped in place");
static_assert(mg::collect_fused_eligible<Glide>(), "continuous actions are supported");
static_assert(mg::collect_fused_eligible<Sized<16, 32>>(), "64-byte State, 32 observations");
static_assert(!mg::collect_fused_eligible<Sized<17, 4>>(), "68-byte State");
static_assert(!mg::collect_fused_eligible<Sized<4, 33>>(), "33 observations");

MG_REGISTER_ENV(Walk)
MG_REGISTER_ENV(TrailWalk)
MG_REGISTER_ENV(Glide)
"""


@pytest.fixture(scope="module")
def user_env_lib(tmp_path_factory):
    import metalgym_b200

    if not metalgym_b200.LIB_PATH.exists():
        pytest.fail("libmetalgym_b200.so not built: run __graft_entry__.build()")
    d = tmp_path_factory.mktemp("user_env")
    src = d / "walk.cu"
    src.write_text(USER_ENV)
    so = d / "libwalk.so"
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--fmad=false",
           "-Xcompiler", "-fPIC", "-shared", "-I", str(ROOT / "include"), str(src), "-o", str(so),
           "-L", str(LIB_DIR), "-lmetalgym_b200", f"-Xlinker=-rpath,{LIB_DIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    metalgym_b200.lib()  # the product library first: the user library registers into it
    return ctypes.CDLL(str(so))


def test_user_environment_registers_with_the_fused_collect(user_env_lib):
    import metalgym_b200
    from metalgym_b200 import EnvOps, _env_has_fused_collect, _env_ops_info

    lib = metalgym_b200.lib()
    names = {lib.mg_env_name(i).decode() for i in range(lib.mg_env_count())}
    assert {"rollout_test_walk", "rollout_test_trail_walk"} <= names
    assert _env_ops_info("rollout_test_walk") == dict(state_bytes=8, action_bytes=4, obs_bytes=8, obs_dim=2,
                                                      act_dim=3, continuous=0)
    assert EnvOps.from_address(lib.mg_env_find(b"rollout_test_walk")).abi_version == lib.mg_version() == 2
    assert _env_has_fused_collect("rollout_test_walk")
    assert not _env_has_fused_collect("rollout_test_trail_walk")
    assert _env_ops_info("rollout_test_glide")["continuous"] == 1
    assert _env_has_fused_collect("rollout_test_glide")


def test_builtin_environments_fused_collect_entries():
    """CartPole and CartPoleContinuous (20-byte states, 4 observations) bring
    the fused kernel; VoxelNav (a 1056-byte state, 40 observations) does not."""
    from metalgym_b200 import _env_has_fused_collect

    assert _env_has_fused_collect("rollout_cartpole")
    assert _env_has_fused_collect("rollout_cartpole_continuous")
    assert not _env_has_fused_collect("rollout_voxelnav")


def test_collect_fused_entry_point_checks_before_the_gpu():
    """mg_env_collect_fused rejects what it cannot run before any CUDA call:
    an unknown environment (MG_ERR_NOT_FOUND), one without the fused kernel
    (MG_ERR_UNSUPPORTED), a depth beyond 4 blocks or missing buffers
    (MG_ERR_ARGUMENT)."""
    import ctypes

    import metalgym_b200
    from metalgym_b200 import CollectFusedArgs

    lib = metalgym_b200.lib()
    a = CollectFusedArgs(parallels=256, horizon=4, layers=2, obs_dim=4, gamma=0.99, lambda_=0.95)
    assert lib.mg_env_collect_fused(b"no_such_env", ctypes.byref(a), None) == 5
    v = CollectFusedArgs(parallels=256, horizon=4, layers=4, obs_dim=40, gamma=0.99, lambda_=0.95)
    assert lib.mg_env_collect_fused(b"rollout_voxelnav", ctypes.byref(v), None) == 3
    assert b"no fused collect kernel" in lib.mg_last_error()
    deep = CollectFusedArgs(parallels=256, horizon=4, layers=5, obs_dim=4)
    assert lib.mg_env_collect_fused(b"rollout_cartpole", ctypes.byref(deep), None) == 1
    assert lib.mg_env_collect_fused(b"rollout_cartpole", ctypes.byref(a), None) == 1  # no buffers
    assert b"null" in lib.mg_last_error()
    # every buffer given, but the head rows (stored as 16-byte vectors) misaligned
    for f in ("w_in", "b_in", "w_head", "states", "done", "rng", "obs_slots", "action_slots", "logp_slots",
              "value_slots", "reward_slots", "done_slots", "adv_slots", "ret_slots"):
        setattr(a, f, 0x10000)
    for i in range(3):
        a.ln_gamma[i] = a.ln_beta[i] = 0x10000
    for i in range(2):
        a.w_up[i] = a.w_down[i] = 0x10000
    a.boot_head = 0x10008
    assert lib.mg_env_collect_fused(b"rollout_cartpole", ctypes.byref(a), None) == 1
    assert b"16-byte aligned" in lib.mg_last_error()
