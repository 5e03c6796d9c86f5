/*
 * rocket_log.h -- the library's single diagnostic channel (same ABI as the
 * reference include/rocket_log.h:39-61).
 *
 * Default sink: ERROR/WARN/INFO to stderr, DEBUG suppressed.  A host installs a
 * callback to take over.  Environment, read once on first use:
 *   ROCKET_LOG_LEVEL = error|warn|info|debug (or 0..3)
 *   ROCKET_DEBUG     -- raises the threshold to DEBUG
 *   ROCKET_LOG_STDERR (non-"0") -- also tee to stderr while a callback is set
 */
#ifndef ROCKET_LOG_H
#define ROCKET_LOG_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    ROCKET_LOG_ERROR = 0,
    ROCKET_LOG_WARN  = 1,
    ROCKET_LOG_INFO  = 2,
    ROCKET_LOG_DEBUG = 3,
} rocket_log_level;

typedef void (*rocket_log_callback)(rocket_log_level level, const char *text, void *user_data);

void             rocket_log_set_callback(rocket_log_callback cb, void *user_data);
void             rocket_log_set_level(rocket_log_level level);
rocket_log_level rocket_log_get_level(void);
void rocket_log(rocket_log_level level, const char *fmt, ...)
#if defined(__GNUC__) || defined(__clang__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;

#define ROCKET_LOGE(...) rocket_log(ROCKET_LOG_ERROR, __VA_ARGS__)
#define ROCKET_LOGW(...) rocket_log(ROCKET_LOG_WARN,  __VA_ARGS__)
#define ROCKET_LOGI(...) rocket_log(ROCKET_LOG_INFO,  __VA_ARGS__)
#define ROCKET_LOGD(...) rocket_log(ROCKET_LOG_DEBUG, __VA_ARGS__)

#ifdef __cplusplus
}
#endif
#endif /* ROCKET_LOG_H */
