// Logging implementation (see include/mpcomm_log.h).
#include "mpcomm_log.h"

#include <pthread.h>
#include <sys/time.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <ctime>

namespace mpcomm {
namespace {

int parse_level() {
    const char *env = std::getenv("MPCOMM_LOG_LEVEL");
    if (!env || !*env) return MPCOMM_LOG_LEVEL_INFO;
    static const struct {
        const char *num, *lo, *up;
        int level;
    } kNames[] = {
        {"0", "error", "ERROR", MPCOMM_LOG_LEVEL_ERROR},
        {"1", "warn", "WARN", MPCOMM_LOG_LEVEL_WARN},
        {"2", "info", "INFO", MPCOMM_LOG_LEVEL_INFO},
        {"3", "debug", "DEBUG", MPCOMM_LOG_LEVEL_DEBUG},
    };
    for (const auto &n : kNames) {
        if (!strcmp(env, n.num) || !strcmp(env, n.lo) || !strcmp(env, n.up))
            return n.level;
    }
    return MPCOMM_LOG_LEVEL_INFO;
}

std::atomic<int> &level_slot() {
    static std::atomic<int> level{parse_level()};
    return level;
}

const char *kTags[] = {"ERROR", "WARN", "INFO", "DEBUG"};

}  // namespace

int mpcomm_get_log_level() { return level_slot().load(std::memory_order_relaxed); }

void mpcomm_reload_log_level() { level_slot().store(parse_level()); }

void mpcomm_log_write(int level, const char *file, int line, int errnum,
                      const char *fmt, ...) {
    char buf[2048];
    struct timeval tv;
    gettimeofday(&tv, nullptr);
    struct tm tm_now;
    localtime_r(&tv.tv_sec, &tm_now);
    const char *base = strrchr(file, '/');
    base = base ? base + 1 : file;
    int lvl = level < 0 ? 0 : (level > 3 ? 3 : level);
    int n = snprintf(buf, sizeof(buf), "[%s] %02d:%02d:%02d.%03d [%04x] %s:%d | ",
                     kTags[lvl], tm_now.tm_hour, tm_now.tm_min, tm_now.tm_sec,
                     static_cast<int>(tv.tv_usec / 1000),
                     static_cast<unsigned>(reinterpret_cast<uintptr_t>(
                                               reinterpret_cast<void *>(pthread_self())) &
                                           0xFFFF),
                     base, line);
    if (n < 0) return;
    size_t used = static_cast<size_t>(n) < sizeof(buf) ? static_cast<size_t>(n) : sizeof(buf) - 1;
    va_list ap;
    va_start(ap, fmt);
    int m = vsnprintf(buf + used, sizeof(buf) - used, fmt, ap);
    va_end(ap);
    if (m > 0) used += static_cast<size_t>(m) < sizeof(buf) - used ? static_cast<size_t>(m)
                                                                   : sizeof(buf) - used - 1;
    if (errnum >= 0) {
        // The PLOG form has no trailing newline in fmt; append the errno text.
        char eb[128];
        const char *es = strerror_r(errnum, eb, sizeof(eb));
        int k = snprintf(buf + used, sizeof(buf) - used, ": %s (errno=%d)\n", es, errnum);
        if (k > 0) used += static_cast<size_t>(k) < sizeof(buf) - used ? static_cast<size_t>(k)
                                                                       : sizeof(buf) - used - 1;
    }
    FILE *fp = level <= MPCOMM_LOG_LEVEL_WARN ? stderr : stdout;
    fwrite(buf, 1, used, fp);
    if (level <= MPCOMM_LOG_LEVEL_WARN) fflush(fp);
}

}  // namespace mpcomm
