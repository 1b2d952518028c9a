/*
 * Minimal Win32 -> POSIX shim so the reference CPU runtime (src/brain_runtime.c,
 * src/brain_runtime_batch.c) compiles unchanged on Linux as an ORACLE.
 *
 * Test infrastructure only: nothing in the product links this header.
 * It covers exactly the Win32 surface those two files touch:
 *   _fseeki64/_ftelli64/__int64, _strnicmp, CreateThread, WaitForSingleObject, WaitForMultipleObjects, CloseHandle,
 *   the TP_WORK thread-pool calls, GetSystemInfo, InterlockedExchange,
 *   QueryPerformance*, GetTickCount64, GetCurrentProcessId, WideCharToMultiByte.
 * Worker count honours ATLAS_REF_THREADS (else the online core count); the
 * reference itself caps GEMV workers at 16 (src/brain_runtime.c:1172).
 */
#ifndef ATLAS_ORACLE_WIN32_SHIM_H
#define ATLAS_ORACLE_WIN32_SHIM_H

#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <strings.h>
#include <time.h>
#include <unistd.h>
#include <wchar.h>
#include <sys/types.h>

typedef int64_t __int64;
typedef int32_t LONG;
typedef uint32_t DWORD;
typedef int BOOL;
typedef void VOID;
typedef void *PVOID;
typedef void *HANDLE;
typedef unsigned int UINT;
#define TRUE 1
#define FALSE 0
#define WINAPI
#define CALLBACK
#define INFINITE 0xFFFFFFFFu
#define WAIT_OBJECT_0 0u
#define CP_UTF8 65001u

#define _fseeki64(f, off, whence) fseeko((f), (off_t)(off), (whence))
#define _ftelli64(f) ((__int64)ftello(f))
#define _strnicmp(a, b, n) strncasecmp((a), (b), (n))

static inline LONG InterlockedExchange(volatile LONG *target, LONG value)
{
    return __atomic_exchange_n(target, value, __ATOMIC_SEQ_CST);
}

typedef struct { DWORD dwNumberOfProcessors; } SYSTEM_INFO;

static inline void GetSystemInfo(SYSTEM_INFO *si)
{
    const char *env = getenv("ATLAS_REF_THREADS");
    long n = env && *env ? strtol(env, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
    si->dwNumberOfProcessors = n > 0 ? (DWORD)n : 1u;
}

/* ---- threads ---- */
typedef DWORD (*LPTHREAD_START_ROUTINE)(void *);
typedef struct {
    pthread_t tid;
    LPTHREAD_START_ROUTINE fn;
    void *arg;
} AtlasShimThread;

static void *atlas_shim_thread_main(void *p)
{
    AtlasShimThread *t = (AtlasShimThread *)p;
    t->fn(t->arg);
    return NULL;
}

static inline HANDLE CreateThread(void *attr, size_t stack, LPTHREAD_START_ROUTINE fn,
                                  void *arg, DWORD flags, DWORD *id)
{
    (void)attr; (void)stack; (void)flags; (void)id;
    AtlasShimThread *t = (AtlasShimThread *)calloc(1, sizeof(*t));
    if (!t) return NULL;
    t->fn = fn;
    t->arg = arg;
    if (pthread_create(&t->tid, NULL, atlas_shim_thread_main, t) != 0) {
        free(t);
        return NULL;
    }
    return t;
}

/* Joins the thread; a joined thread is marked so CloseHandle only frees it. */
static inline DWORD WaitForSingleObject(HANDLE h, DWORD ms)
{
    (void)ms;
    AtlasShimThread *t = (AtlasShimThread *)h;
    if (t && t->fn) { pthread_join(t->tid, NULL); t->fn = NULL; }
    return WAIT_OBJECT_0;
}

static inline DWORD WaitForMultipleObjects(DWORD n, HANDLE *hs, BOOL all, DWORD ms)
{
    (void)all;
    for (DWORD i = 0; i < n; ++i) WaitForSingleObject(hs[i], ms);
    return WAIT_OBJECT_0;
}

static inline BOOL CloseHandle(HANDLE h)
{
    WaitForSingleObject(h, INFINITE);
    free(h);
    return TRUE;
}

/* ---- thread pool (one pthread per submitted work item) ---- */
typedef void *PTP_CALLBACK_INSTANCE;
typedef struct AtlasShimWork *PTP_WORK;
typedef void (*PTP_WORK_CALLBACK)(PTP_CALLBACK_INSTANCE, PVOID, PTP_WORK);
struct AtlasShimWork {
    pthread_t tid;
    PTP_WORK_CALLBACK cb;
    PVOID ctx;
    int running;
};

static void *atlas_shim_work_main(void *p)
{
    PTP_WORK w = (PTP_WORK)p;
    w->cb(NULL, w->ctx, w);
    return NULL;
}

static inline PTP_WORK CreateThreadpoolWork(PTP_WORK_CALLBACK cb, PVOID ctx, void *env)
{
    (void)env;
    PTP_WORK w = (PTP_WORK)calloc(1, sizeof(*w));
    if (w) { w->cb = cb; w->ctx = ctx; }
    return w;
}

static inline void SubmitThreadpoolWork(PTP_WORK w)
{
    if (pthread_create(&w->tid, NULL, atlas_shim_work_main, w) == 0) w->running = 1;
    else w->cb(NULL, w->ctx, w);
}

static inline void WaitForThreadpoolWorkCallbacks(PTP_WORK w, BOOL cancel)
{
    (void)cancel;
    if (w->running) { pthread_join(w->tid, NULL); w->running = 0; }
}

static inline void CloseThreadpoolWork(PTP_WORK w) { free(w); }

/* ---- clocks and ids ---- */
typedef union { struct { DWORD LowPart; LONG HighPart; } u; int64_t QuadPart; } LARGE_INTEGER;

static inline BOOL QueryPerformanceCounter(LARGE_INTEGER *c)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    c->QuadPart = (int64_t)ts.tv_sec * 1000000000LL + ts.tv_nsec;
    return TRUE;
}

static inline BOOL QueryPerformanceFrequency(LARGE_INTEGER *f)
{
    f->QuadPart = 1000000000LL;
    return TRUE;
}

static inline uint64_t GetTickCount64(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000u + (uint64_t)(ts.tv_nsec / 1000000);
}

static inline DWORD GetCurrentProcessId(void) { return (DWORD)getpid(); }

/* UTF-16 argv conversion is never exercised by the oracle (it calls the
   runtime's functions directly); wchar_t is 32-bit here, so copy code points
   that fit in ASCII and reject the rest. */
static inline int WideCharToMultiByte(UINT cp, DWORD flags, const wchar_t *src, int n,
                                      char *dst, int cap, const char *dflt, BOOL *used)
{
    (void)cp; (void)flags; (void)dflt; (void)used;
    int len = 0;
    if (n < 0) { while (src[len]) ++len; ++len; } else len = n;
    if (!dst) return len;
    if (cap < len) return 0;
    for (int i = 0; i < len; ++i) {
        if ((unsigned)src[i] > 127u) return 0;
        dst[i] = (char)src[i];
    }
    return len;
}

#endif
