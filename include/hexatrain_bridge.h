/*
 * hexatrain_bridge.h -- the host-app bridge of the reference
 * (app/src/main/cpp/native_bridge.cpp, JNI class
 * com.yuubinnkyoku.phonelm.NativeBridge) restated over libhexatrain_b200.so.
 *
 * The reference's Kotlin host calls NativeBridge.native* (NativeBridge.kt:
 * 7-182) and receives KEY=VALUE report strings.  These functions are the
 * JNI-free core of that bridge: hexatrain_b200/jni/native_bridge_b200.cpp
 * wraps each one in the reference's Java_com_yuubinnkyoku_phonelm_
 * NativeBridge_* symbol where a JDK's jni.h is available; C, C++ and Python
 * hosts call them directly.  Reports are valid until the next bridge call
 * on the same thread.
 */
#ifndef HEXATRAIN_BRIDGE_H
#define HEXATRAIN_BRIDGE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Arguments of nativeRunExecutionMode (native_bridge.cpp:252-276), in
 * order.  Served modes (training_engine.h:10-115):
 *   32 QNN_HTP_MLP_FULL_STEP, 33 QNN_HTP_MLP_FULL_STEP_BENCHMARK,
 *   35 QNN_HTP_MLP_FULL_STEP_FAIL_EXECUTE (host failure injection at
 *      execute 37, as the reference), with batch_size=B, dimension=I,
 *      hidden_dimension=H, output_dimension=O, sample_count samples,
 *      steps = epochs > 0 ? sample_count/B*epochs : steps;
 *   99 QNN_HTP_TINY_LANGUAGE_MODEL_GENERIC: sample_count=T,
 *      output_dimension=V, dimension=D, hidden_dimension=FFN, epochs=L,
 *      measured_steps=H, steps=Adam updates, batch_size sequences per
 *      step, training_stability_mode, and an NPRTCKPTV2 checkpoint written
 *      to diagnostic_checkpoint_dir (resumed from when
 *      diagnostic_resume_step > 0).
 * Any other mode reports status=FAILED with
 * failure_classification=UNSUPPORTED_EXECUTION_MODE. */
typedef struct {
    int32_t execution_mode;
    int32_t batch_size, dimension, hidden_dimension, output_dimension;
    int32_t steps, warmup_steps;
    float learning_rate;
    int64_t seed;
    int32_t sample_count, epochs, measured_steps, correctness_interval;
    int32_t benchmark_mode, seed_selection_mode, training_stability_mode;
    int32_t depth_pair_init_mode, checkpoint_selection_mode, diagnostic_trajectory;
    const char* diagnostic_checkpoint_dir;
    int32_t diagnostic_resume_step, diagnostic_checkpoint_interval;
    /* progress lines (the Kotlin onNativeProgress callback); may be NULL */
    void (*progress)(void* context, const char* line);
    void* progress_context;
} hx_bridge_run;

/* nativeGetEnvironmentInfo (native_bridge.cpp:140-156). */
const char* hx_bridge_environment_report(void);
/* nativeGetQnnStatus (:158-170): whether a B200-class device can run the
 * library. */
const char* hx_bridge_status_report(void);
/* nativeRunExecutionMode (:252-373): one run at a time per process. */
const char* hx_bridge_run_execution_mode(const hx_bridge_run* run);
/* nativeRequestStop / nativeClearStop (:1100-1124): a stop requested during
 * a run ends it after the current step. */
void hx_bridge_request_stop(void);
void hx_bridge_clear_stop(void);

#ifdef __cplusplus
}
#endif
#endif /* HEXATRAIN_BRIDGE_H */
