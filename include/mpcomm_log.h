// Leveled logging for mpcomm.
//
// Level comes from MPCOMM_LOG_LEVEL, read once: 0/error, 1/warn, 2/info
// (default), 3/debug — the same scale as reference include/mpcomm_log.h:44-70.
// Line format: "[LEVEL] HH:MM:SS.mmm [tid] file:line | message", DEBUG/INFO to
// stdout and WARN/ERROR to stderr; MPCOMM_PLOG_ERROR appends strerror(errno).
// Unlike the reference, each line is formatted into one buffer and written
// with a single fwrite so lines from worker threads never interleave.
#ifndef MPCOMM_B200_INCLUDE_MPCOMM_LOG_H_
#define MPCOMM_B200_INCLUDE_MPCOMM_LOG_H_

#include <cerrno>
#include <cstdarg>
#include <cstring>

namespace mpcomm {

enum MPCommLogLevel {
    MPCOMM_LOG_LEVEL_ERROR = 0,
    MPCOMM_LOG_LEVEL_WARN = 1,
    MPCOMM_LOG_LEVEL_INFO = 2,
    MPCOMM_LOG_LEVEL_DEBUG = 3,
};

// Parsed once (thread-safe static init).
int mpcomm_get_log_level();
// Re-reads MPCOMM_LOG_LEVEL (tests).
void mpcomm_reload_log_level();
// Formats and writes one line. `errnum` >= 0 appends ": strerror (errno=N)".
void mpcomm_log_write(int level, const char *file, int line, int errnum,
                      const char *fmt, ...)
    __attribute__((format(printf, 5, 6)));

}  // namespace mpcomm

#define MPCOMM_LOG_AT_(lvl, errnum, fmt, ...)                                   \
    do {                                                                        \
        if (mpcomm::mpcomm_get_log_level() >= (lvl))                            \
            mpcomm::mpcomm_log_write((lvl), __FILE__, __LINE__, (errnum), fmt,  \
                                     ##__VA_ARGS__);                            \
    } while (0)

#define MPCOMM_LOG_DEBUG(fmt, ...) \
    MPCOMM_LOG_AT_(mpcomm::MPCOMM_LOG_LEVEL_DEBUG, -1, fmt, ##__VA_ARGS__)
#define MPCOMM_LOG_INFO(fmt, ...) \
    MPCOMM_LOG_AT_(mpcomm::MPCOMM_LOG_LEVEL_INFO, -1, fmt, ##__VA_ARGS__)
#define MPCOMM_LOG_WARN(fmt, ...) \
    MPCOMM_LOG_AT_(mpcomm::MPCOMM_LOG_LEVEL_WARN, -1, fmt, ##__VA_ARGS__)
#define MPCOMM_LOG_ERROR(fmt, ...) \
    MPCOMM_LOG_AT_(mpcomm::MPCOMM_LOG_LEVEL_ERROR, -1, fmt, ##__VA_ARGS__)
#define MPCOMM_PLOG_ERROR(fmt, ...)                                             \
    do {                                                                        \
        int mpcomm_saved_errno_ = errno;                                        \
        mpcomm::mpcomm_log_write(mpcomm::MPCOMM_LOG_LEVEL_ERROR, __FILE__,      \
                                 __LINE__, mpcomm_saved_errno_, fmt,            \
                                 ##__VA_ARGS__);                                \
    } while (0)

#endif  // MPCOMM_B200_INCLUDE_MPCOMM_LOG_H_
