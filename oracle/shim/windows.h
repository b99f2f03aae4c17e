/*
 * Minimal POSIX stand-in for the two Win32 timing calls that the reference's
 * weight provider uses (src/kq_weight_provider.c:53-55,392-394,461-476 of
 * Kestrel-Q).  It lets the reference's hot-path C compile on Linux so that it
 * can serve as the CPU oracle and CPU baseline.  Test infrastructure only.
 */
#ifndef KQ_ORACLE_WINDOWS_SHIM_H
#define KQ_ORACLE_WINDOWS_SHIM_H

#include <stdint.h>
#include <time.h>

typedef union _LARGE_INTEGER {
    struct {
        uint32_t LowPart;
        int32_t HighPart;
    } u;
    long long QuadPart;
} LARGE_INTEGER;

static inline int QueryPerformanceFrequency(LARGE_INTEGER *frequency) {
    frequency->QuadPart = 1000000000LL;
    return 1;
}

static inline int QueryPerformanceCounter(LARGE_INTEGER *counter) {
    struct timespec now;
    if (clock_gettime(CLOCK_MONOTONIC, &now) != 0) {
        return 0;
    }
    counter->QuadPart = (long long)now.tv_sec * 1000000000LL + now.tv_nsec;
    return 1;
}

#endif
