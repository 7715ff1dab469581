/*
 * Linux stand-ins for the handful of Win32 APIs that the Minima reference's
 * host support files (util.c, arena.c, tokenizer.c) call.  Test
 * infrastructure only: it lets those files compile unmodified with gcc so
 * that the reference decoder can serve as the parity oracle.
 *
 * Semantics follow the documented Win32 contracts closely enough for the
 * reference's use: VirtualAlloc(MEM_RESERVE) reserves address space,
 * VirtualAlloc(MEM_COMMIT) on a sub-range makes it readable/writable and
 * zero-filled, VirtualFree(MEM_RELEASE) with size 0 releases the whole
 * reservation.
 */
#ifndef MINIMA_ORACLE_COMPAT_WINDOWS_H
#define MINIMA_ORACLE_COMPAT_WINDOWS_H

#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <errno.h>
#include <sched.h>
#include <stdio.h>
#include <time.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

typedef uint32_t DWORD;
typedef int32_t LONG;
typedef int BOOL;
typedef void* LPVOID;

#define MEM_COMMIT   0x1000u
#define MEM_RESERVE  0x2000u
#define MEM_RELEASE  0x8000u
#define PAGE_NOACCESS  0x01u
#define PAGE_READWRITE 0x04u
#define INVALID_FILE_ATTRIBUTES ((DWORD)0xFFFFFFFFu)
#define FILE_ATTRIBUTE_DIRECTORY 0x10u
#define MOVEFILE_REPLACE_EXISTING 0x1u
#define MOVEFILE_WRITE_THROUGH 0x8u

typedef struct { DWORD dwPageSize; } SYSTEM_INFO;
typedef union { struct { DWORD LowPart; LONG HighPart; } u; int64_t QuadPart; } LARGE_INTEGER;
typedef union { struct { DWORD LowPart; DWORD HighPart; }; uint64_t QuadPart; } ULARGE_INTEGER;
typedef struct {
    DWORD dwFileAttributes;
    DWORD nFileSizeHigh;
    DWORD nFileSizeLow;
} WIN32_FILE_ATTRIBUTE_DATA;
typedef enum { GetFileExInfoStandard = 0 } GET_FILEEX_INFO_LEVELS;

/* Reservations keep their total length in a header page so that
   VirtualFree(base, 0, MEM_RELEASE) can unmap without a side table. */
static inline size_t compat_page_size(void) {
    long p = sysconf(_SC_PAGESIZE);
    return p > 0 ? (size_t)p : 4096u;
}

static inline LPVOID VirtualAlloc(LPVOID addr, size_t size, DWORD type, DWORD protect) {
    const size_t page = compat_page_size();
    if (type & MEM_RESERVE) {
        if (size > SIZE_MAX - page) return NULL;
        uint8_t* raw = (uint8_t*)mmap(NULL, size + page, PROT_NONE,
            MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
        if (raw == (uint8_t*)MAP_FAILED) return NULL;
        if (mprotect(raw, page, PROT_READ | PROT_WRITE) != 0) {
            munmap(raw, size + page);
            return NULL;
        }
        *(size_t*)raw = size + page;
        uint8_t* base = raw + page;
        if (protect == PAGE_READWRITE &&
            mprotect(base, size, PROT_READ | PROT_WRITE) != 0) {
            munmap(raw, size + page);
            return NULL;
        }
        return base;
    }
    if (type & MEM_COMMIT) {
        if (!addr) return NULL;
        uintptr_t start = (uintptr_t)addr & ~(uintptr_t)(page - 1);
        uintptr_t end = ((uintptr_t)addr + size + page - 1) & ~(uintptr_t)(page - 1);
        int prot = protect == PAGE_NOACCESS ? PROT_NONE : PROT_READ | PROT_WRITE;
        if (mprotect((void*)start, end - start, prot) != 0) return NULL;
        return addr;
    }
    return NULL;
}

static inline BOOL VirtualFree(LPVOID addr, size_t size, DWORD type) {
    (void)size;
    if (!addr || !(type & MEM_RELEASE)) return 0;
    uint8_t* raw = (uint8_t*)addr - compat_page_size();
    return munmap(raw, *(size_t*)raw) == 0;
}

static inline void GetSystemInfo(SYSTEM_INFO* info) {
    info->dwPageSize = (DWORD)compat_page_size();
}

static inline DWORD GetLastError(void) { return (DWORD)errno; }

static inline LONG InterlockedCompareExchange(volatile LONG* dst, LONG xchg, LONG cmp) {
    return __sync_val_compare_and_swap(dst, cmp, xchg);
}

static inline LONG InterlockedExchange(volatile LONG* dst, LONG value) {
    return __atomic_exchange_n(dst, value, __ATOMIC_SEQ_CST);
}

static inline void Sleep(DWORD ms) {
    if (ms == 0) { sched_yield(); return; }
    struct timespec ts = { (time_t)(ms / 1000u), (long)(ms % 1000u) * 1000000L };
    nanosleep(&ts, NULL);
}

static inline DWORD GetFileAttributesA(const char* path) {
    struct stat st;
    if (stat(path, &st) != 0) return INVALID_FILE_ATTRIBUTES;
    return S_ISDIR(st.st_mode) ? FILE_ATTRIBUTE_DIRECTORY : 0x80u;
}

static inline BOOL GetFileAttributesExA(const char* path, GET_FILEEX_INFO_LEVELS level,
    void* out) {
    (void)level;
    struct stat st;
    if (stat(path, &st) != 0) return 0;
    WIN32_FILE_ATTRIBUTE_DATA* fad = (WIN32_FILE_ATTRIBUTE_DATA*)out;
    fad->dwFileAttributes = S_ISDIR(st.st_mode) ? FILE_ATTRIBUTE_DIRECTORY : 0x80u;
    fad->nFileSizeHigh = (DWORD)((uint64_t)st.st_size >> 32);
    fad->nFileSizeLow = (DWORD)((uint64_t)st.st_size & 0xFFFFFFFFu);
    return 1;
}

static inline BOOL QueryPerformanceFrequency(LARGE_INTEGER* f) {
    f->QuadPart = 1000000000LL;
    return 1;
}

static inline BOOL QueryPerformanceCounter(LARGE_INTEGER* t) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    t->QuadPart = (int64_t)ts.tv_sec * 1000000000LL + ts.tv_nsec;
    return 1;
}

static inline BOOL MoveFileExA(const char* from, const char* to, DWORD flags) {
    (void)flags;
    return rename(from, to) == 0;
}

/* checkpoint.c: archive slots and the atomic save. */
#define FALSE 0
#define TRUE 1
#define MAX_PATH 260
#define ERROR_FILE_NOT_FOUND 2u   /* == ENOENT, which GetLastError returns here */
#define ERROR_PATH_NOT_FOUND 3u
#define _TRUNCATE ((size_t)-1)

#include <stdarg.h>
/* _snprintf_s(buf, size, _TRUNCATE, ...): -1 when the output was truncated. */
static inline int compat_snprintf_s(char* buf, size_t size, size_t count, const char* fmt, ...) {
    (void)count;
    va_list ap;
    va_start(ap, fmt);
    const int n = vsnprintf(buf, size, fmt, ap);
    va_end(ap);
    return (n < 0 || (size_t)n >= size) ? -1 : n;
}
#define _snprintf_s compat_snprintf_s

static inline BOOL DeleteFileA(const char* path) { return unlink(path) == 0; }

static inline BOOL CopyFileA(const char* from, const char* to, BOOL fail_if_exists) {
    if (fail_if_exists && access(to, F_OK) == 0) return 0;
    FILE* in = fopen(from, "rb");
    if (!in) return 0;
    FILE* out = fopen(to, "wb");
    if (!out) { fclose(in); return 0; }
    char buf[65536];
    size_t n;
    BOOL ok = 1;
    while ((n = fread(buf, 1, sizeof(buf), in)) > 0)
        if (fwrite(buf, 1, n, out) != n) { ok = 0; break; }
    if (ferror(in)) ok = 0;
    fclose(in);
    if (fclose(out) != 0) ok = 0;
    return ok;
}

#endif
