/*
 * NVTX injection library for the tests: the NVTX v3 client inside libsparc_b200.so loads it
 * through NVTX_INJECTION64_PATH on its first call and hands it the core callback table; it
 * replaces the range push / pop entries with functions that record "push:<name>" and "pop" lines
 * in a buffer that the test reads with nvtx_recorder_log(). No GPU is involved.
 */
#include <stddef.h>
#include <string.h>

#include <nvtx3/nvToolsExt.h> /* the injection interface types (NvtxExportTableCallbacks, ...) */

static char g_log[1 << 16];
static size_t g_len;

static void record(const char* a, const char* b) {
  const size_t na = strlen(a), nb = b ? strlen(b) : 0;
  if (g_len + na + nb + 2 >= sizeof(g_log)) return;
  memcpy(g_log + g_len, a, na);
  g_len += na;
  if (b) {
    memcpy(g_log + g_len, b, nb);
    g_len += nb;
  }
  g_log[g_len++] = '\n';
  g_log[g_len] = '\0';
}

static int range_push_a(const char* message) {
  record("push:", message);
  return 0;
}

static int range_pop(void) {
  record("pop", NULL);
  return 0;
}

int InitializeInjectionNvtx2(NvtxGetExportTableFunc_t get_export_table) {
  const NvtxExportTableCallbacks* cb = (const NvtxExportTableCallbacks*)get_export_table(NVTX_ETID_CALLBACKS);
  NvtxFunctionTable table = NULL;
  unsigned int size = 0;
  if (cb == NULL || !cb->GetModuleFunctionTable(NVTX_CB_MODULE_CORE, &table, &size) || table == NULL) return 0;
  if (size <= NVTX_CBID_CORE_RangePop) return 0;
  *table[NVTX_CBID_CORE_RangePushA] = (NvtxFunctionPointer)range_push_a;
  *table[NVTX_CBID_CORE_RangePop] = (NvtxFunctionPointer)range_pop;
  return 1;
}

const char* nvtx_recorder_log(void) { return g_log; }
