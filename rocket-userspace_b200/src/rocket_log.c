/*
 * rocket_log.c -- the library's single diagnostic channel.  Same ABI and
 * environment contract as the reference src/rocket_log.c:66-129: a host
 * callback takes over when installed; the threshold comes from
 * ROCKET_LOG_LEVEL / ROCKET_DEBUG; ROCKET_LOG_STDERR tees to stderr.
 */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <strings.h>
#include <pthread.h>

#include "rocket_log.h"

static rocket_log_callback g_cb;
static void *g_ud;
static int g_level = -1;
static int g_tee = -1;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void log_init(void)
{
    int lvl = ROCKET_LOG_INFO;
    const char *e = getenv("ROCKET_LOG_LEVEL");
    if (e && *e) {
        if (!strcasecmp(e, "error") || !strcmp(e, "0")) lvl = ROCKET_LOG_ERROR;
        else if (!strcasecmp(e, "warn") || !strcmp(e, "1")) lvl = ROCKET_LOG_WARN;
        else if (!strcasecmp(e, "info") || !strcmp(e, "2")) lvl = ROCKET_LOG_INFO;
        else if (!strcasecmp(e, "debug") || !strcmp(e, "3")) lvl = ROCKET_LOG_DEBUG;
    }
    if (getenv("ROCKET_DEBUG") && lvl < ROCKET_LOG_DEBUG) lvl = ROCKET_LOG_DEBUG;
    if (g_level < 0) g_level = lvl;
    const char *t = getenv("ROCKET_LOG_STDERR");
    g_tee = (t && *t && strcmp(t, "0") != 0) ? 1 : 0;
}

void rocket_log_set_callback(rocket_log_callback cb, void *user_data)
{
    g_cb = cb;
    g_ud = user_data;
}

void rocket_log_set_level(rocket_log_level level)
{
    pthread_once(&g_once, log_init);
    g_level = (int)level;
}

rocket_log_level rocket_log_get_level(void)
{
    pthread_once(&g_once, log_init);
    return (rocket_log_level)g_level;
}

void rocket_log(rocket_log_level level, const char *fmt, ...)
{
    pthread_once(&g_once, log_init);
    if ((int)level > g_level) return;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (g_cb) {
        g_cb(level, buf, g_ud);
        if (g_tee) fputs(buf, stderr);
    } else {
        fputs(buf, stderr);
    }
}
