/*
 * Linux stand-in for <sys/sysctl.h> (removed from glibc).  TEST INFRASTRUCTURE
 * ONLY.  The reference asks sysctlbyname("hw.activecpu") for its row-chunk
 * count (quantize.c:460); answer with the online CPU count.
 */
#ifndef SS_ORACLE_SHIM_SYSCTL_H
#define SS_ORACLE_SHIM_SYSCTL_H
#include <stddef.h>
#include <stdint.h>
#include <unistd.h>
static inline int sysctlbyname(const char *name, void *oldp, size_t *oldlenp,
                               void *newp, size_t newlen) {
    (void)name; (void)newp; (void)newlen;
    if (!oldp || !oldlenp || *oldlenp < sizeof(int32_t)) return -1;
    *(int32_t *)oldp = (int32_t)sysconf(_SC_NPROCESSORS_ONLN);
    return 0;
}
#endif
