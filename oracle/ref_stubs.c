/* ref_stubs.c -- link stubs for building the reference's CPU-side code as a checker (oracle/_ref).
 *
 * TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles the ork-driver translation units that build on
 * x86 (the NPU-submit and NEON-only ones do not) into oracle/_ref/libork_ref.so so the tests can run the
 * reference's own offline CPU path (ork_npu_init_offline -> ork_i8_mm_pack/run, ork_i4_mm_pack/run,
 * ork_i4a8_pack_cpu_blob, ork_i4a8_mm_load). The symbols below are only reached on device paths, which an
 * offline context never takes; they abort so that an unexpected device call is loud. Three are real:
 *   orki_io_ok        -- an ioctl on the offline fd (-1) fails, as the real one would (returns -1);
 *   ork_npu_free      -- an offline context owns nothing but its own allocation;
 *   ork_pack_format_version -- the on-disk format token, 1 (include/ork_npu.h:37 in ork-driver).
 * This file deliberately includes no reference header: the abort stubs take no arguments and are
 * resolved by name only. */
#include <stdint.h>
#include <stdlib.h>

int orki_io_ok(int fd, unsigned long req, void *arg, const char *what, int may_fail)
{
    (void)fd; (void)req; (void)arg; (void)what; (void)may_fail;
    return -1;
}
void ork_npu_free(void *ctx) { free(ctx); }
uint32_t ork_pack_format_version(void) { return 1u; }
void *orki_npu_ctx = NULL;

#define ORC_ABORT_STUB(name) void name(void) { abort(); }
ORC_ABORT_STUB(ork_ctx_fd_reap)
ORC_ABORT_STUB(ork_dyn_begin_colsplit)
ORC_ABORT_STUB(ork_dyn_end)
ORC_ABORT_STUB(ork_dyn_grouped_end)
ORC_ABORT_STUB(ork_dyn_seq_end)
ORC_ABORT_STUB(ork_f16_npu_add)
ORC_ABORT_STUB(ork_f16_npu_ewmul)
ORC_ABORT_STUB(ork_f16_npu_mul_perchan)
ORC_ABORT_STUB(ork_i4_dyn_begin_mc)
ORC_ABORT_STUB(ork_i4_dyn_begin_mc_grouped)
ORC_ABORT_STUB(ork_i4_mm_run_chain)
ORC_ABORT_STUB(ork_i8_dyn_begin_seq_mc)
ORC_ABORT_STUB(ork_i8_mm_run_chain)
ORC_ABORT_STUB(ork_kmsg)
ORC_ABORT_STUB(ork_npu_chain_progs)
ORC_ABORT_STUB(ork_npu_dump_state)
ORC_ABORT_STUB(ork_npu_init_orkd)
ORC_ABORT_STUB(ork_npu_mode_reset)
ORC_ABORT_STUB(ork_npu_reap_stuck)
ORC_ABORT_STUB(orki_act)
ORC_ABORT_STUB(orki_act_opt)
ORC_ABORT_STUB(orki_check_extent)
ORC_ABORT_STUB(orki_check_overlap)
ORC_ABORT_STUB(orki_dyn_begin_mc_impl)
ORC_ABORT_STUB(orki_i4_bchain_try)
ORC_ABORT_STUB(orki_i4_hcap)
ORC_ABORT_STUB(orki_i4_run_experts_bchain_db)
ORC_ABORT_STUB(orki_i8_chain_fullk_mcap)
ORC_ABORT_STUB(orki_i8_run_chain_impl)
ORC_ABORT_STUB(orki_rknpu_submit_ioctl)
ORC_ABORT_STUB(orki_setrn)
ORC_ABORT_STUB(orki_slice_rescue_or_refuse)
ORC_ABORT_STUB(orki_submit1)
ORC_ABORT_STUB(orki_submit1_db)
ORC_ABORT_STUB(orki_validate_regcmd)
ORC_ABORT_STUB(orki_warn_if_governor_parked)
/* npu.c names these NEON intrinsics without <arm_neon.h> on x86, on device-only paths. */
ORC_ABORT_STUB(vaddq_f32)
ORC_ABORT_STUB(vaddq_s32)
ORC_ABORT_STUB(vld1q_f32)
ORC_ABORT_STUB(vld1q_s32)
ORC_ABORT_STUB(vst1q_f32)
ORC_ABORT_STUB(vst1q_s32)
