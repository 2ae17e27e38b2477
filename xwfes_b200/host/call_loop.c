/* call_loop.c -- a native caller of ftc_backend_matmul for the end-to-end
 * benchmark.
 *
 * The reference's engine is C++: each decode step calls IBackend::matmul
 * once per projection from a plain loop (ft/src/engine.cpp:514-516, 569,
 * 588; the interface at ft/include/ft/backend.h:28-29), and every call
 * returns with y on the host.  ftc_call_loop makes the same sequence of
 * synchronous calls through the C ABI from native code, so a Python
 * harness can time the per-call cost an engine sees without an interpreter
 * between the calls.  The ABI entry is passed in as a function pointer (the
 * address ctypes resolved in the already loaded libftcuda.so), so this
 * library links against nothing.
 *
 * Returns 0, or the first non-zero status of a call (the loop stops there;
 * ftc_last_error() holds the message). */
#include <stdint.h>

typedef int (*ftc_matmul_fn)(void* be, const float* x, int64_t M, int64_t K, const void* w,
                             int dtype, int64_t N, float* y);

int ftc_call_loop(void* fn, void* be, int n_calls, const float* const* x, const int64_t* M,
                  const int64_t* K, const void* const* w, const int* dtype, const int64_t* N,
                  float* const* y, int reps) {
    const ftc_matmul_fn mm = (ftc_matmul_fn)fn;
    if (!mm || !be || n_calls < 0 || reps < 0) return -1;
    for (int r = 0; r < reps; ++r)
        for (int i = 0; i < n_calls; ++i) {
            const int rc = mm(be, x[i], M[i], K[i], w[i], dtype[i], N[i], y[i]);
            if (rc) return rc;
        }
    return 0;
}
