/* NVTX injection library for tests/test_nvtx.py: TEST INFRASTRUCTURE ONLY.
 *
 * The NVTX runtime inside libuq_b200 loads the library named by
 * NVTX_INJECTION64_PATH at its first NVTX call and calls
 * InitializeInjectionNvtx2, which points the domain create / push / pop
 * slots of the CORE2 callback table at the recorders below.  Each event is
 * appended as one line to the file named by UQ_NVTX_RECORD:
 *     "domain <name>"   a domain was created
 *     "+<message>"      a range was pushed
 *     "-"               the innermost range was popped
 */
#include <stdio.h>
#include <stdlib.h>

#include <nvtx3/nvToolsExt.h>

static struct nvtxDomainRegistration_st *const rec_handle = (struct nvtxDomainRegistration_st *)(void *)&rec_handle;

static void rec_put(const char *tag, const char *msg) {
    const char *path = getenv("UQ_NVTX_RECORD");
    if (!path) return;
    FILE *f = fopen(path, "a");
    if (!f) return;
    fprintf(f, "%s%s\n", tag, msg ? msg : "");
    fclose(f);
}

static nvtxDomainHandle_t rec_domain_create(const char *name) {
    rec_put("domain ", name);
    return rec_handle;
}

static int rec_push(nvtxDomainHandle_t d, const nvtxEventAttributes_t *a) {
    (void)d;
    rec_put("+", (a && a->messageType == NVTX_MESSAGE_TYPE_ASCII) ? a->message.ascii : "?");
    return 0;
}

static int rec_pop(nvtxDomainHandle_t d) {
    (void)d;
    rec_put("-", "");
    return 0;
}

int InitializeInjectionNvtx2(NvtxGetExportTableFunc_t get_table) {
    const NvtxExportTableCallbacks *cb = (const NvtxExportTableCallbacks *)get_table(NVTX_ETID_CALLBACKS);
    NvtxFunctionTable t = 0;
    unsigned int n = 0;
    if (!cb || !cb->GetModuleFunctionTable(NVTX_CB_MODULE_CORE2, &t, &n) || !t) return 0;
    if (n <= NVTX_CBID_CORE2_DomainCreateA) return 0;
    *t[NVTX_CBID_CORE2_DomainCreateA] = (NvtxFunctionPointer)rec_domain_create;
    *t[NVTX_CBID_CORE2_DomainRangePushEx] = (NvtxFunctionPointer)rec_push;
    *t[NVTX_CBID_CORE2_DomainRangePop] = (NvtxFunctionPointer)rec_pop;
    return 1;
}
