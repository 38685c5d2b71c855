"""Host-side helpers of the per-kernel step profiler (vm_c_b200/utils/step_profile.py)."""
from vm_c_b200.utils.step_profile import family, merge_max, report, short


def test_kernel_names_and_families():
    assert short("void vmc::(anonymous namespace)::gemm_qd_kernel<1, 64>(CUtensorMap_st, vmc::GemmArgs)") == \
        "gemm_qd_kernel<1, 64>"
    assert short("void vmc::rs_norm_ag_kernel<2, (bool)0>(vmc::RsArgs)") == "rs_norm_ag_kernel<2, (bool)0>"
    assert short("ncclDevKernel_AllReduce_Sum_f32_RING_LL(ncclDevKernelArgsStorage<4096ul>)") == \
        "ncclDevKernel_AllReduce_Sum_f32_RING_LL"
    assert family("gemm_qd_kernel<1, 64>") == "gemm"
    assert family("attn_prefill_tc_kernel") == "attention"
    assert family("rs_norm_ag_kernel<2, (bool)0>") == "rs_norm_ag"
    assert family("ncclDevKernel_AllReduce_Sum_f32_RING_LL") == "nccl"
    assert family("add_rmsnorm_vec_kernel") == "norm_rope_embed"
    assert family("Memcpy HtoD (Pinned -> Device)") == "other"


def test_merge_is_max_over_ranks_and_report_sums_families():
    a = {"gemm_qd_kernel<1, 64>": [100.0, 4.0], "rs_norm_ag_kernel<2, (bool)0>": [30.0, 2.0]}
    b = {"gemm_qd_kernel<1, 64>": [120.0, 4.0], "attn_decode_kernel<128, 0>": [10.0, 1.0]}
    m = merge_max([a, b])
    assert m["gemm_qd_kernel<1, 64>"] == [120.0, 4.0]
    assert m["attn_decode_kernel<128, 0>"] == [10.0, 1.0] and m["rs_norm_ag_kernel<2, (bool)0>"] == [30.0, 2.0]
    lines = report("decode", m, 200.0)
    assert "200.0 us per step" in lines[0]
    assert "kernel time per step 160.0 us" in lines[1]
    assert lines[2].split()[0] == "gemm" and "120.0 us" in lines[2]
