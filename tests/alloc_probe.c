/*
 * alloc_probe.c -- test infrastructure for tests/test_zz_no_alloc.py.
 *
 * Counts CUDA driver API calls that allocate memory (any cuMemAlloc*,
 * cuMemCreate, cuMemHostAlloc, cuMemPoolCreate, cuMemAllocFromPool*) made
 * by any code in the process, through CUPTI's callback API: every CUDA
 * runtime, the static one linked into libmxfp8.so included, reaches the
 * driver, and CUPTI sees each driver call on entry.  Free device memory
 * (cudaMemGetInfo) cannot show a 256-byte cudaMalloc: the driver serves it
 * from memory it already holds.
 *
 *   alloc_probe_start()        subscribe (once); returns 0 or a CUPTI error
 *   alloc_probe_count()        allocation calls seen since the start
 *   alloc_probe_last_name()    the function name of the last one seen
 */
#include <cupti.h>
#include <string.h>

static volatile long g_count = 0;
static const char* volatile g_last = "";
static CUpti_SubscriberHandle g_sub;
static int g_started = 0;

static int is_allocation(const char* name) {
    if (!name) return 0;
    return strncmp(name, "cuMemAlloc", 10) == 0 || strncmp(name, "cuMemCreate", 11) == 0 ||
           strncmp(name, "cuMemHostAlloc", 14) == 0 || strncmp(name, "cuMemPoolCreate", 15) == 0;
}

static void CUPTIAPI on_api(void* userdata, CUpti_CallbackDomain domain, CUpti_CallbackId cbid,
                            const void* cbdata) {
    (void)userdata;
    (void)cbid;
    if (domain != CUPTI_CB_DOMAIN_DRIVER_API) return;
    const CUpti_CallbackData* d = (const CUpti_CallbackData*)cbdata;
    if (d->callbackSite != CUPTI_API_ENTER || !is_allocation(d->functionName)) return;
    __sync_fetch_and_add(&g_count, 1);
    g_last = d->functionName;
}

int alloc_probe_start(void) {
    if (g_started) return 0;
    CUptiResult r = cuptiSubscribe(&g_sub, (CUpti_CallbackFunc)on_api, 0);
    if (r != CUPTI_SUCCESS) return (int)r;
    r = cuptiEnableDomain(1, g_sub, CUPTI_CB_DOMAIN_DRIVER_API);
    if (r != CUPTI_SUCCESS) return (int)r;
    g_started = 1;
    return 0;
}

long alloc_probe_count(void) { return g_count; }

const char* alloc_probe_last_name(void) { return g_last; }
