/* Test-only syscall fault injection for kvsnap_b200/csrc/io.cpp, linked with
   -Wl,--wrap=pwrite,--wrap=pread,--wrap=fdatasync. Each wrapper counts its calls
   and, while a plan for it is armed, fails, shortens or stalls the next calls.
   While io_stall(1) holds, every pread and pwrite waits at its entry, so a test
   can count how many transfers a pool lets run at once. */
#include <errno.h>
#include <pthread.h>
#include <sys/types.h>
#include <unistd.h>

static pthread_mutex_t stall_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t stall_cv = PTHREAD_COND_INITIALIZER;
static int stalled = 0, inside = 0, peak = 0;

void io_stall(int on) {
    pthread_mutex_lock(&stall_mu);
    stalled = on;
    if (!on) pthread_cond_broadcast(&stall_cv);
    pthread_mutex_unlock(&stall_mu);
}

/* Transfers waiting at the stall now; the most seen at once (reset by the call). */
int io_inside(void) {
    pthread_mutex_lock(&stall_mu);
    int n = inside;
    pthread_mutex_unlock(&stall_mu);
    return n;
}

int io_peak(void) {
    pthread_mutex_lock(&stall_mu);
    int n = peak;
    peak = 0;
    pthread_mutex_unlock(&stall_mu);
    return n;
}

static void stall_point(void) {
    pthread_mutex_lock(&stall_mu);
    if (++inside > peak) peak = inside;
    while (stalled) pthread_cond_wait(&stall_cv, &stall_mu);
    --inside;
    pthread_mutex_unlock(&stall_mu);
}

enum { PWRITE = 0, PREAD = 1, FDATASYNC = 2 };
enum { FAIL = 1, SHORT = 2, NOTHING = 3 };

static int plan_call = -1, plan_kind = 0, plan_left = 0, plan_errno = 0;
static int calls[3];

ssize_t __real_pwrite(int, const void*, size_t, off_t);
ssize_t __real_pread(int, void*, size_t, off_t);
int __real_fdatasync(int);

void io_fault(int call, int kind, int times, int err) {
    plan_call = call; plan_kind = kind; plan_left = times; plan_errno = err;
}

int io_calls(int call) {
    int n = calls[call];
    calls[call] = 0;
    return n;
}

static int armed(int call) {
    calls[call]++;
    if (plan_call != call || plan_left <= 0) return 0;
    plan_left--;
    return plan_kind;
}

ssize_t __wrap_pwrite(int fd, const void* data, size_t size, off_t offset) {
    stall_point();
    switch (armed(PWRITE)) {
    case FAIL: errno = plan_errno; return -1;
    case SHORT: return __real_pwrite(fd, data, size ? 1 : 0, offset);
    case NOTHING: return 0;
    }
    return __real_pwrite(fd, data, size, offset);
}

ssize_t __wrap_pread(int fd, void* data, size_t size, off_t offset) {
    stall_point();
    switch (armed(PREAD)) {
    case FAIL: errno = plan_errno; return -1;
    case SHORT: return __real_pread(fd, data, size ? 1 : 0, offset);
    case NOTHING: return 0;
    }
    return __real_pread(fd, data, size, offset);
}

int __wrap_fdatasync(int fd) {
    if (armed(FDATASYNC) == FAIL) { errno = plan_errno; return -1; }
    return __real_fdatasync(fd);
}
