// runtime.cu - library-wide state: error channel, precision mode, device info.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace cg {

namespace {
int g_status = OK;
char g_msg[512] = "";
// CNGPT_CUDA_PRECISION = tf32 | 3xtf32 | fp32 selects the starting mode (the
// reference's own test programs have no other way to choose it)
int initial_precision() {
    const char *e = getenv("CNGPT_CUDA_PRECISION");
    if (!e) return PREC_3XTF32;
    if (!strcmp(e, "tf32")) return PREC_TF32;
    if (!strcmp(e, "fp32")) return PREC_FP32;
    return PREC_3XTF32;
}
int g_precision = initial_precision();
int g_sms = 0;
}  // namespace

void set_last_error(int status, const char *fmt, ...) {
    g_status = status;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    if (getenv("CNGPT_CUDA_VERBOSE")) fprintf(stderr, "libcngpt_cuda: %s\n", g_msg);
}

int last_status() { return g_status; }
const char *last_message() { return g_msg; }

int check_device_error() {
    int (*readers[])() = {gemm_take_dev_error, attn_take_dev_error, tp_take_dev_error,
                            attn_tc_take_dev_error, mk_take_dev_error};
    for (auto rd : readers) {
        int code = rd();
        if (code < 0) {
            set_last_error(ERR_CUDA, "reading the device error word failed");
            return ERR_CUDA;
        }
        if (code != 0) {
            set_last_error(ERR_DEVICE_WAIT, "device-side bounded wait gave up (site %d)", code);
            return ERR_DEVICE_WAIT;
        }
    }
    return OK;
}

int set_wait_limit_ns(unsigned long long ns) {
    int (*setters[])(unsigned long long) = {gemm_set_wait_limit, attn_set_wait_limit, tp_set_wait_limit,
                                            attn_tc_set_wait_limit, mk_set_wait_limit};
    for (auto set : setters)
        if (set(ns) != 0) {
            set_last_error(ERR_CUDA, "setting the device wait limit failed");
            return ERR_CUDA;
        }
    return OK;
}

int precision() { return g_precision; }
void set_precision(int p) { g_precision = p; }

int num_sms() {
    if (g_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

}  // namespace cg
