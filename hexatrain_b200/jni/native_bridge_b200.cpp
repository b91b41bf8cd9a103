// native_bridge_b200.cpp -- the reference's JNI surface
// (app/src/main/cpp/native_bridge.cpp, Kotlin NativeBridge.kt:7-182) for
// the training-step path, over the bridge core of libhexatrain_b200.so
// (include/hexatrain_bridge.h).  Each function only converts JNI values and
// forwards; the behaviour lives in the core.
//
// Built by hexatrain_b200/build.py into libhexatrain_b200_jni.so when a
// JDK's jni.h is found (JAVA_HOME, or HX_JNI_INCLUDE); the Kotlin host then
// loads it in place of the reference's libphonelm.so for these entry
// points.  Entry points of the reference that drive the on-device
// Nicopedia corpus, MNN backends or HTP probes have no counterpart here.
#include <jni.h>

#include <string>

#include "hexatrain_bridge.h"

namespace {

jstring to_java(JNIEnv* env, const char* text) { return env->NewStringUTF(text ? text : ""); }

struct Progress {
    JNIEnv* env;
    jobject callback;
    jmethodID method;
};

void forward_progress(void* context, const char* line) {
    auto* p = static_cast<Progress*>(context);
    if (!p || !p->method) return;
    jstring s = p->env->NewStringUTF(line);
    p->env->CallVoidMethod(p->callback, p->method, s);
    if (p->env->ExceptionCheck()) p->env->ExceptionClear();
    p->env->DeleteLocalRef(s);
}

}  // namespace

extern "C" JNIEXPORT jstring JNICALL
Java_com_yuubinnkyoku_phonelm_NativeBridge_nativeGetEnvironmentInfo(JNIEnv* env, jobject) {
    return to_java(env, hx_bridge_environment_report());
}

extern "C" JNIEXPORT jstring JNICALL
Java_com_yuubinnkyoku_phonelm_NativeBridge_nativeGetQnnStatus(JNIEnv* env, jobject) {
    return to_java(env, hx_bridge_status_report());
}

extern "C" JNIEXPORT jstring JNICALL Java_com_yuubinnkyoku_phonelm_NativeBridge_nativeRunExecutionMode(
    JNIEnv* env, jobject, jint executionMode, jint batchSize, jint dimension, jint hiddenDimension,
    jint outputDimension, jint steps, jint warmupSteps, jfloat learningRate, jlong seed, jint sampleCount,
    jint epochs, jint measuredSteps, jint correctnessInterval, jboolean benchmarkMode, jint seedSelectionMode,
    jint trainingStabilityMode, jint depthPairInitMode, jint checkpointSelectionMode,
    jboolean diagnosticTrajectory, jstring diagnosticCheckpointDir, jint diagnosticResumeStep,
    jint diagnosticCheckpointInterval, jobject progressCallback) {
    std::string dir;
    if (diagnosticCheckpointDir) {
        const char* chars = env->GetStringUTFChars(diagnosticCheckpointDir, nullptr);
        if (chars) {
            dir = chars;
            env->ReleaseStringUTFChars(diagnosticCheckpointDir, chars);
        }
    }
    Progress progress{env, progressCallback, nullptr};
    if (progressCallback) {
        jclass cls = env->GetObjectClass(progressCallback);
        if (cls) {
            progress.method = env->GetMethodID(cls, "onNativeProgress", "(Ljava/lang/String;)V");
            env->DeleteLocalRef(cls);
        }
        if (env->ExceptionCheck()) {
            env->ExceptionClear();
            progress.method = nullptr;
        }
    }
    hx_bridge_run run{};
    run.execution_mode = executionMode;
    run.batch_size = batchSize;
    run.dimension = dimension;
    run.hidden_dimension = hiddenDimension;
    run.output_dimension = outputDimension;
    run.steps = steps;
    run.warmup_steps = warmupSteps;
    run.learning_rate = learningRate;
    run.seed = seed;
    run.sample_count = sampleCount;
    run.epochs = epochs;
    run.measured_steps = measuredSteps;
    run.correctness_interval = correctnessInterval;
    run.benchmark_mode = benchmarkMode ? 1 : 0;
    run.seed_selection_mode = seedSelectionMode;
    run.training_stability_mode = trainingStabilityMode;
    run.depth_pair_init_mode = depthPairInitMode;
    run.checkpoint_selection_mode = checkpointSelectionMode;
    run.diagnostic_trajectory = diagnosticTrajectory ? 1 : 0;
    run.diagnostic_checkpoint_dir = dir.c_str();
    run.diagnostic_resume_step = diagnosticResumeStep;
    run.diagnostic_checkpoint_interval = diagnosticCheckpointInterval;
    run.progress = progress.method ? forward_progress : nullptr;
    run.progress_context = &progress;
    return to_java(env, hx_bridge_run_execution_mode(&run));
}

extern "C" JNIEXPORT void JNICALL Java_com_yuubinnkyoku_phonelm_NativeBridge_nativeRequestStop(JNIEnv*, jobject) {
    hx_bridge_request_stop();
}

extern "C" JNIEXPORT void JNICALL Java_com_yuubinnkyoku_phonelm_NativeBridge_nativeClearStop(JNIEnv*, jobject) {
    hx_bridge_clear_stop();
}

extern "C" JNIEXPORT jint JNI_OnLoad(JavaVM*, void*) { return JNI_VERSION_1_6; }
