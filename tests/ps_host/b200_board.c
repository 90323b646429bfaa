/* Platform layer that runs the reference's unchanged PS firmware
 * (src/software/main.c, generation.c, tokenizer.c, utf8_stream.c, built with
 * QWEN_HOST_SIM) on a host with a B200: it supplies the functions the
 * firmware calls through its BSP headers (the src/software/tests/shim headers) and
 * routes the accelerator's CSR window and ACT_IN embedding copies to
 * libqwen_b200's CSR emulation (include/qwen_b200.h), which runs the model
 * on the GPU.
 *
 *   Xil_Out64 / Xil_In64 at QWEN_CSR_BASE + off -> qwen_b200_csr_write / read
 *   sim_embedding(token, row)  (main.c copy_embedding) -> qwen_b200_embedding
 *   sim_clear()                (main.c reset_context)  -> qwen_b200_clear
 *   qwen_board_prepare()       opens the handle and loads the SD package
 *   f_* (FatFs)                files under $SIM_SD ("0:/X" -> "$SIM_SD/X"); the
 *                              model assets, which the firmware would copy into
 *                              DDR windows, are accepted without being read:
 *                              the engine loaded them into HBM already
 *   XUartPs_* / usleep / XTime  stdin / stdout, the host clock
 *
 * Environment: SIM_SD (folder holding QWEN25/), QWEN_B200_DEVICE (default 0).
 * Test harness; it holds no model arithmetic.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "ff.h"
#include "xil_io.h"
#include "xiltimer.h"
#include "xuartps.h"
#include "board_parameters.h"
#include "qwen_b200.h"

static qwen_b200 *board;

static const char *sd_root(void) {
    const char *root = getenv("SIM_SD");
    return root ? root : ".";
}

void Xil_DCacheDisable(void) {}

int qwen_board_prepare(void) {
    qwen_b200_config cfg;
    qwen_b200_default_config(&cfg);
    const char *dev = getenv("QWEN_B200_DEVICE");
    cfg.device = dev ? atoi(dev) : 0;
    cfg.max_context = QWEN_KV_CAPACITY; /* the firmware's KV capacity (256) */
    if (qwen_b200_open(&cfg, &board)) return -1;
    if (qwen_b200_load_assets(board, sd_root())) {
        fprintf(stderr, "libqwen_b200: %s\n", qwen_b200_last_error(board));
        return -1;
    }
    return 0;
}

void Xil_Out64(UINTPTR address, uint64_t value) {
    qwen_b200_csr_write(board, (unsigned)(address - QWEN_CSR_BASE), value);
}
uint64_t Xil_In64(UINTPTR address) { return qwen_b200_csr_read(board, (unsigned)(address - QWEN_CSR_BASE)); }
void sim_embedding(unsigned token, unsigned row) { qwen_b200_embedding(board, token, row); }
void sim_clear(void) { qwen_b200_clear(board); }

void usleep(unsigned us) {
    struct timespec t = {us / 1000000u, (long)(us % 1000000u) * 1000L};
    nanosleep(&t, NULL);
}
void XTime_GetTime(XTime *out) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    *out = (XTime)t.tv_sec * 1000000u + (XTime)(t.tv_nsec / 1000); /* COUNTS_PER_SECOND = 1e6 */
}

XUartPs_Config *XUartPs_LookupConfig(uintptr_t base) {
    static XUartPs_Config c;
    c.BaseAddress = base;
    return &c;
}
int XUartPs_CfgInitialize(XUartPs *u, XUartPs_Config *c, uintptr_t base) {
    (void)u;
    (void)c;
    (void)base;
    return 0;
}
int XUartPs_SetBaudRate(XUartPs *u, unsigned baud) {
    (void)u;
    return baud == 115200 ? 0 : -1;
}
void XUartPs_SetOperMode(XUartPs *u, unsigned mode) {
    (void)u;
    (void)mode;
}
void XUartPs_SendByte(uintptr_t base, unsigned char c) {
    (void)base;
    putchar(c);
}
unsigned char XUartPs_RecvByte(uintptr_t base) {
    (void)base;
    const int c = getchar();
    if (c == EOF) {
        fflush(stdout);
        if (board) qwen_b200_close(board);
        exit(0);
    }
    return (unsigned char)c;
}

/* FatFs over the host file system. */
FRESULT f_mount(FATFS *fs, const char *path, int now) {
    (void)fs;
    (void)path;
    (void)now;
    return FR_OK;
}
FRESULT f_open(FIL *f, const char *path, int flags) {
    memset(f, 0, sizeof(*f));
    for (unsigned i = 0; i < QWEN_ASSET_COUNT; ++i)
        if (!strcmp(path, assets[i].filename)) {
            f->asset = 1;
            f->size = assets[i].bytes;
            return FR_OK;
        }
    char name[4096];
    snprintf(name, sizeof(name), "%s/%s", sd_root(), strncmp(path, "0:/", 3) ? path : path + 3);
    f->handle = fopen(name, (flags & FA_WRITE) ? "r+b" : "rb");
    if (!f->handle && (flags & FA_OPEN_ALWAYS)) f->handle = fopen(name, "w+b");
    if (!f->handle) return 1;
    fseek(f->handle, 0, SEEK_END);
    f->size = (uint64_t)ftell(f->handle);
    rewind(f->handle);
    return FR_OK;
}
FRESULT f_close(FIL *f) {
    if (f->handle) fclose(f->handle);
    f->handle = NULL;
    return FR_OK;
}
FRESULT f_read(FIL *f, void *out, UINT n, UINT *got) {
    if (f->asset) { /* already resident in HBM */
        *got = n;
        f->offset += n;
        return FR_OK;
    }
    *got = (UINT)fread(out, 1, n, f->handle);
    return ferror(f->handle) ? 1 : FR_OK;
}
FRESULT f_write(FIL *f, const void *data, UINT n, UINT *written) {
    *written = (UINT)fwrite(data, 1, n, f->handle);
    f->size = (uint64_t)ftell(f->handle);
    return *written == n ? FR_OK : 1;
}
FRESULT f_sync(FIL *f) { return fflush(f->handle) ? 1 : FR_OK; }
FRESULT f_lseek(FIL *f, uint64_t offset) { return fseek(f->handle, (long)offset, SEEK_SET) ? 1 : FR_OK; }
