/* A C99 host of libtitan_b200 that needs no GPU: the header compiles as plain C, the
 * library links, and the host-side entries answer through the C ABI alone.
 *
 *   host_check <dir>   writes <dir>/kernels.tune; prints one "ok <check>" line per check
 *                      and exits 0, or prints "FAIL <check>: <detail>" and exits 1. */
#include <stdio.h>
#include <string.h>

#include "titan_b200.h"

static int failures = 0;

static void check(int ok, const char* what, const char* detail) {
  if (ok) {
    printf("ok %s\n", what);
  } else {
    printf("FAIL %s: %s\n", what, detail ? detail : "");
    ++failures;
  }
}

int main(int argc, char** argv) {
  char path[4096], buf[8192], key[1024];
  size_t len = 0, records = 0, ignored = 0;
  tb_tune_store* store = NULL;
  tb_tensor none[1];
  tb_tensor out;
  tb_event* ev = NULL;
  tb_status st;
  if (argc != 2) return 2;

  check(tb_version() != NULL && tb_version()[0] != '\0', "version", NULL);

  /* FIPS 180-2 appendix B.1: SHA-256("abc"). */
  tb_sha256_hex("abc", 3, buf);
  check(strcmp(buf, "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad") == 0, "sha256", buf);

  st = tb_tune_canonical_json("{ \"b\": [1, 2.50], \"a\": \"\\u00e9\" }", buf, sizeof buf, &len);
  check(st == TB_OK && strcmp(buf, "{\"a\":\"\\u00e9\",\"b\":[1,2.5]}") == 0, "canonical_json", buf);

  snprintf(path, sizeof path, "%s/kernels.tune", argv[1]);
  st = tb_tune_open(path, &store);
  check(st == TB_OK, "tune_open", tb_last_error_detail());
  st = tb_tune_insert(store, "{\"operator\": \"gemm\", \"shape\": \"[8,8]\"}", "{\"candidate\": \"gemm_bf16_tn\"}");
  check(st == TB_OK, "tune_insert", tb_last_error_detail());
  st = tb_tune_flush(store);
  check(st == TB_OK, "tune_flush", tb_last_error_detail());
  tb_tune_release(store);
  store = NULL;
  st = tb_tune_open(path, &store);
  check(st == TB_OK, "tune_reopen", tb_last_error_detail());
  st = tb_tune_get(store, "{\"shape\":\"[8,8]\",\"operator\":\"gemm\"}", buf, sizeof buf, &len);
  check(st == TB_OK && strcmp(buf, "{\"candidate\":\"gemm_bf16_tn\"}") == 0, "tune_get", buf);
  st = tb_tune_stats(store, &records, &ignored);
  check(st == TB_OK && records == 1 && ignored == 0, "tune_stats", NULL);
  st = tb_tune_record(store, 0, key, sizeof key, &len, buf, sizeof buf, &len);
  check(st == TB_OK && strcmp(key, "{\"operator\":\"gemm\",\"shape\":\"[8,8]\"}") == 0, "tune_record", key);
  st = tb_tune_get(store, "{\"operator\":\"softmax\"}", buf, sizeof buf, &len);
  check(st == TB_OK && len == 0, "tune_miss", NULL);
  /* Too small a buffer reports the length needed. */
  st = tb_tune_record(store, 0, key, 4, &len, buf, sizeof buf, &records);
  check(st == TB_ERR_INVALID && len == strlen("{\"operator\":\"gemm\",\"shape\":\"[8,8]\"}"), "short_buffer", NULL);
  tb_tune_release(store);

  st = tb_graph_compile(
      "{\"inputs\":[0,1,2],\"outputs\":[5],"
      "\"values\":{\"0\":{\"dtype\":\"BF16\",\"shape\":[8,16]},\"1\":{\"dtype\":\"BF16\",\"shape\":[32,16]},"
      "\"2\":{\"dtype\":\"F32\",\"shape\":[32]},\"3\":{\"dtype\":\"BF16\",\"shape\":[8,32]},"
      "\"4\":{\"dtype\":\"BF16\",\"shape\":[8,32]},\"5\":{\"dtype\":\"BF16\",\"shape\":[8,32]}},"
      "\"nodes\":[{\"id\":10,\"operator\":\"gemm\",\"inputs\":[0,1],\"outputs\":[3],\"attrs\":{\"transpose_rhs\":true}},"
      "{\"id\":11,\"operator\":\"broadcast.add\",\"inputs\":[3,2],\"outputs\":[4],\"attrs\":{}},"
      "{\"id\":12,\"operator\":\"gelu\",\"inputs\":[4],\"outputs\":[5],\"attrs\":{}}]}",
      "compile", buf, sizeof buf, &len);
  check(st == TB_OK && strstr(buf, "\"operator\":\"gemm.bias_act\"") && strstr(buf, "\"activation\":\"gelu\""),
        "graph_compile", buf);
  st = tb_graph_compile("{\"inputs\":[],\"outputs\":[7],\"values\":{},\"nodes\":[]}", NULL, buf, sizeof buf, &len);
  check(st == TB_ERR_INVALID && strstr(buf, "value 7 has no TensorSpec"), "graph_error", buf);

  memset(none, 0, sizeof none);
  memset(&out, 0, sizeof out);
  st = tb_execute(NULL, NULL, "layer_norm", none, 1, &out, NULL, 0, &ev);
  check(st == TB_ERR_UNSUPPORTED && strcmp(tb_last_error_operation(), "contract") == 0, "execute_route",
        tb_last_error_detail());

  return failures ? 1 : 0;
}
