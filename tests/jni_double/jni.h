/* Test double of a JDK's jni.h: just the types and JNIEnv calls that
 * hexatrain_b200/jni/native_bridge_b200.cpp uses, dispatching through a
 * function table as the real header does.  It lets the CPU tests compile
 * the JNI bridge and check its exported symbols where no JDK is installed;
 * it is never used to build the shipped library. */
#ifndef HX_TEST_JNI_DOUBLE_H
#define HX_TEST_JNI_DOUBLE_H
#include <stdint.h>

#define JNIEXPORT __attribute__((visibility("default")))
#define JNICALL
#define JNI_VERSION_1_6 0x00010006

typedef int32_t jint;
typedef int64_t jlong;
typedef float jfloat;
typedef uint8_t jboolean;
typedef struct _jobject* jobject;
typedef jobject jclass;
typedef jobject jstring;
typedef struct _jmethodID* jmethodID;
struct JavaVM;
struct JNIEnv;

struct JNIFunctionTable {
    jstring (*NewStringUTF)(JNIEnv*, const char*);
    const char* (*GetStringUTFChars)(JNIEnv*, jstring, jboolean*);
    void (*ReleaseStringUTFChars)(JNIEnv*, jstring, const char*);
    jclass (*GetObjectClass)(JNIEnv*, jobject);
    jmethodID (*GetMethodID)(JNIEnv*, jclass, const char*, const char*);
    void (*CallVoidMethodOneArg)(JNIEnv*, jobject, jmethodID, jobject);
    jboolean (*ExceptionCheck)(JNIEnv*);
    void (*ExceptionClear)(JNIEnv*);
    void (*DeleteLocalRef)(JNIEnv*, jobject);
};

struct JNIEnv {
    const JNIFunctionTable* functions;
    jstring NewStringUTF(const char* s) { return functions->NewStringUTF(this, s); }
    const char* GetStringUTFChars(jstring s, jboolean* copy) { return functions->GetStringUTFChars(this, s, copy); }
    void ReleaseStringUTFChars(jstring s, const char* c) { functions->ReleaseStringUTFChars(this, s, c); }
    jclass GetObjectClass(jobject o) { return functions->GetObjectClass(this, o); }
    jmethodID GetMethodID(jclass c, const char* n, const char* sig) { return functions->GetMethodID(this, c, n, sig); }
    void CallVoidMethod(jobject o, jmethodID m, jobject arg) { functions->CallVoidMethodOneArg(this, o, m, arg); }
    jboolean ExceptionCheck() { return functions->ExceptionCheck(this); }
    void ExceptionClear() { functions->ExceptionClear(this); }
    void DeleteLocalRef(jobject o) { functions->DeleteLocalRef(this, o); }
};
#endif
