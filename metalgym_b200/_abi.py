"""ctypes signatures of every function declared in include/metalgym_b200.h.

tests/test_abi.py checks that this table and the header declare the same set
of functions and that the built library exports all of them.
"""
import ctypes as C

P = C.c_void_p
I = C.c_int
U = C.c_uint32
F = C.c_float
U64 = C.c_uint64
S = C.c_char_p
PI = C.POINTER(C.c_int)
PF = C.POINTER(C.c_float)

SIGNATURES = {
    # runtime
    "mg_last_error": (S, []),
    "mg_version": (I, []),
    "mg_device_status": (I, [I, PI]),
    # GEMM
    "mg_gemm_bf16": (I, [P, I, I, P, I, I, I, I, I, I, P, I, P, I, I, P]),
    "mg_block_forward": (I, [P, P, P, P, P, P, P, P, P, I, I, I, P]),
    "mg_gemm_bf16_resid_layernorm": (I, [P, I, P, I, I, I, I, I, P, P, P, P, P, P, P]),
    "mg_gemm_rows_resid_layernorm": (I, [P, I, P, I, I, I, I, P, P, P, P, P, P, P]),
    "mg_gemm_rows_layernorm_backward": (I, [P, I, P, I, I, I, I, P, P, P, P, P, P, P]),
    "mg_gemm_rows_splits": (I, [I]),
    "mg_head_tail": (I, [P, P, P, P, P, P, P, P, P, P, I, I, F, F, F, P, P, P, P, P, P, P]),
    "mg_block_cluster_forward_input": (I, [P, I] + [P] * 16 + [I, P]),
    "mg_block_cluster_forward": (I, [P, P, P, P, P, P, P, P, P, P, I, P]),
    "mg_block_cluster_backward": (I, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I, P, I, P]),
    "mg_gemm_bf16_tiled": (I, [P, I, I, P, I, I, I, I, I, I, P, I, P, I, I, I, I, P]),
    # environments
    "mg_env_register": (I, [P]),
    "mg_env_find": (P, [S]),
    "mg_env_count": (I, []),
    "mg_env_name": (S, [I]),
    "mg_env_init": (I, [S, P, P, P, I, U, U, P]),
    "mg_env_step": (I, [S, P, P, P, P, P, P, P, I, P]),
    "mg_env_run_random": (I, [S, P, P, P, P, P, P, I, I, I, I, P]),
    "mg_env_collect_fused": (I, [S, P, P]),
    "mg_env_collect_step": (I, [S, P, P, P, P, P, P, P, P, P, P, P, I, P]),
    # policy kernels
    "mg_input_forward": (I, [P, P, P, P, I, I, I, P]),
    "mg_input_forward_layernorm": (I, [P, P, P, P, P, P, P, P, P, I, I, I, P]),
    "mg_input_backward_partials": (I, [P, P, P, I, I, I, P]),
    "mg_input_backward_num_partials": (I, [I, I, I]),
    "mg_layernorm_forward": (I, [P, P, P, P, P, P, I, I, P]),
    "mg_layernorm_backward": (I, [P, P, P, P, P, P, I, I, P]),
    "mg_layernorm_backward_num_partials": (I, [I]),
    "mg_sample_categorical": (I, [P, P, P, P, P, I, I, P]),
    "mg_sample_gaussian": (I, [P, P, P, P, P, P, I, I, P]),
    "mg_policy_loss": (I, [P, P, P, P, P, P, P, P, I, I, F, F, F, P]),
    "mg_gaussian_loss": (I, [P, P, P, P, P, P, P, P, P, P, I, I, F, F, F, P]),
    "mg_gaussian_loss_num_partials": (I, [I]),
    "mg_gae": (I, [P, P, P, P, P, P, I, I, I, F, F, P]),
    "mg_advantage_stats": (I, [P, P, I, I, P]),
    "mg_reduce_partials": (I, [P, C.c_int64, I, C.c_int64, P, I, P, P]),
    "mg_reduce_partials_num_norm_partials": (I, [C.c_int64]),
    "mg_adam_step": (I, [P, P, P, P, P, P, I, C.c_int64, F, F, F, F, P, P]),
    "mg_stats_mean": (I, [P, I, P, P]),
    # sessions
    "mg_gym_create": (I, [S, I, U, U, I, C.POINTER(P)]),
    "mg_gym_destroy": (I, [P]),
    "mg_gym_info": (I, [P, P]),
    "mg_gym_run": (I, [P, P, P, I]),
    "mg_gym_run_random": (I, [P, I, I]),
    "mg_gym_buffer": (I, [P, I, C.POINTER(P), C.POINTER(C.c_size_t)]),
    "mg_gym_download": (I, [P, I, P, C.c_size_t]),
    "mg_gym_upload": (I, [P, I, P, C.c_size_t]),
    "mg_gym_stream": (I, [P, C.POINTER(P)]),
    "mg_gym_synchronize": (I, [P]),
    "mg_ppo_create": (I, [P, I, I, I, F, I, U, C.POINTER(P)]),
    "mg_ppo_destroy": (I, [P]),
    "mg_ppo_info": (I, [P, P]),
    "mg_ppo_param_info": (I, [P, I, C.POINTER(U64), C.POINTER(U), PI]),
    "mg_ppo_collect": (I, [P]),
    "mg_ppo_train": (I, [P, I]),
    "mg_ppo_train_slot": (I, [P, I]),
    "mg_ppo_p2p_handle": (I, [P, P]),
    "mg_ppo_p2p_open": (I, [P, P, I, I]),
    "mg_ppo_save": (I, [P, S]),
    "mg_ppo_load": (I, [P, S]),
    "mg_ppo_set_minibatch_rows": (I, [P, I]),
    "mg_ppo_minibatch_rows": (I, [P, PI]),
    "mg_ppo_set_collect_fused": (I, [P, I]),
    "mg_ppo_set_allreduce_overlap": (I, [P, I]),
    "mg_ppo_set_comm_timeout": (I, [P, F]),
    "mg_ppo_phase_ms": (I, [P, PF]),
    "mg_ppo_collect_fused": (I, [P, PI]),
    "mg_ppo_set_fused_minibatch": (I, [P, I]),
    "mg_set_tile_trace": (I, [P]),
    "mg_ppo_act_greedy": (I, [P, I, P]),
    "mg_ppo_fused_minibatch": (I, [P, PI]),
    "mg_ppo_train_rows": (I, [P, P, U]),
    "mg_minibatch_rows": (I, [P, U, U, U64, P]),
    "mg_ppo_forward": (I, [P]),
    "mg_ppo_last_stats": (I, [P, P]),
    "mg_ppo_set_hyper": (I, [P, F, F, F, F, F, F]),
    "mg_ppo_get_hyper": (I, [P, P]),
    "mg_ppo_set_log_std": (I, [P, F]),
    "mg_ppo_log_std": (I, [P, I, PF]),
    "mg_ppo_step_counter": (I, [P, PF]),
    "mg_ppo_set_step_counter": (I, [P, F]),
    "mg_ppo_buffer": (I, [P, I, I, C.POINTER(P), C.POINTER(C.c_size_t)]),
    "mg_ppo_download": (I, [P, I, I, P, C.c_size_t]),
    "mg_ppo_upload": (I, [P, I, I, P, C.c_size_t]),
    "mg_ppo_graph_kernels": (I, [P, P]),
    "mg_ppo_set_comm": (I, [P, P, I, I]),
    # NCCL / host memory
    "mg_comm_unique_id": (I, [P]),
    "mg_comm_init": (I, [I, I, P, I, C.POINTER(P)]),
    "mg_comm_destroy": (I, [P]),
    "mg_comm_abort": (I, [P]),
    "mg_allreduce_sum_f32": (I, [P, C.c_size_t, P, P]),
    "mg_host_alloc": (I, [C.c_size_t, C.POINTER(P)]),
    "mg_host_free": (I, [P]),
    # no-allocation variant
    "mg_weight_grad_noalloc": (I, [P, P, I, I, I, I, I, P, P]),
}
