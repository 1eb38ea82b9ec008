// The three example environments of the reference (CartPole,
// CartPoleContinuous, VoxelNav), registered under their reference kernel
// names, and the tanh-squashed CartPoleContinuous of the BASELINE text
// (rollout_cartpole_continuous_tanh). Compiled with --fmad=false (see metalgym_b200/build.py).
#include "metalgym/envs/cartpole.h"
#include "metalgym/envs/cartpole_continuous.h"
#include "metalgym/envs/voxelnav.h"
#include "metalgym/register_env.cuh"

MG_REGISTER_ENV(CartPole)
MG_REGISTER_ENV(CartPoleContinuous)
MG_REGISTER_ENV(CartPoleContinuousTanh)
MG_REGISTER_ENV(VoxelNav)
