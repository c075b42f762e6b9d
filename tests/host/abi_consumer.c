/*
 * A plain C99 client of libfuton_cuda, as cgo compiles one: both headers
 * must build as C, and the library must link and run from C without any
 * Python. Tokenises its arguments with the native tokenizer through the
 * batch entry point and prints one line of ids per text; no GPU is needed.
 *
 *   abi_consumer VOCAB MAX_SEQ_LEN TEXT...
 *
 * It sizes the ids buffer too small on purpose first: the batch call must
 * fail with FUTON_EINVAL and report the exact total in cu_seqlens.
 */
#include "futon_cuda.h"
#include "futon_tokenizer.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char* slurp(const char* path, size_t* len) {
  FILE* f = fopen(path, "rb");
  char* buf;
  long n;
  if (!f) return NULL;
  if (fseek(f, 0, SEEK_END) != 0 || (n = ftell(f)) < 0 || fseek(f, 0, SEEK_SET) != 0) {
    fclose(f);
    return NULL;
  }
  buf = (char*)malloc((size_t)n + 1);
  if (buf && fread(buf, 1, (size_t)n, f) != (size_t)n) {
    free(buf);
    buf = NULL;
  }
  fclose(f);
  *len = (size_t)n;
  return buf;
}

int main(int argc, char** argv) {
  char err[512];
  size_t vlen = 0, total = 0;
  char *vocab, *text;
  int64_t* off;
  int32_t *cu, *ids;
  int ntexts, max_len, i, j, rc;
  futon_tokenizer_cfg cfg;
  futon_tokenizer* tok = NULL;

  if (argc < 3) {
    fprintf(stderr, "usage: abi_consumer VOCAB MAX_SEQ_LEN TEXT...\n");
    return 2;
  }
  vocab = slurp(argv[1], &vlen);
  if (!vocab) {
    fprintf(stderr, "cannot read %s\n", argv[1]);
    return 2;
  }
  memset(&cfg, 0, sizeof cfg);
  cfg.do_lower_case = 1;
  cfg.tokenize_chinese_chars = 1;
  if (futon_tokenizer_create(vocab, vlen, &cfg, &tok, err, sizeof err) != FUTON_OK) {
    fprintf(stderr, "create: %s\n", err);
    return 1;
  }
  free(vocab);
  printf("devices %d vocab %d pad %d\n", futon_cuda_device_count(),
         futon_tokenizer_vocab_size(tok), futon_tokenizer_pad_id(tok));

  max_len = atoi(argv[2]);
  ntexts = argc - 3;
  off = (int64_t*)calloc((size_t)ntexts + 1, sizeof *off);
  cu = (int32_t*)calloc((size_t)ntexts + 1, sizeof *cu);
  for (i = 0; i < ntexts; ++i) total += strlen(argv[3 + i]);
  text = (char*)malloc(total + 1);
  for (i = 0; i < ntexts; ++i) {
    size_t n = strlen(argv[3 + i]);
    memcpy(text + off[i], argv[3 + i], n);
    off[i + 1] = off[i] + (int64_t)n;
  }

  ids = (int32_t*)malloc(sizeof *ids);
  rc = futon_tokenizer_encode_batch(tok, text, off, ntexts, max_len, 0, ids, 1, cu, err,
                                    sizeof err);
  if (ntexts > 0 && rc != FUTON_EINVAL) {
    fprintf(stderr, "a 1-id buffer was accepted (rc %d)\n", rc);
    return 1;
  }
  free(ids);
  ids = (int32_t*)malloc(sizeof *ids * ((size_t)cu[ntexts] + 1));
  rc = futon_tokenizer_encode_batch(tok, text, off, ntexts, max_len, 0, ids,
                                    (int64_t)cu[ntexts], cu, err, sizeof err);
  if (rc != FUTON_OK) {
    fprintf(stderr, "encode_batch: %s\n", err);
    return 1;
  }
  for (i = 0; i < ntexts; ++i) {
    for (j = cu[i]; j < cu[i + 1]; ++j) printf(j > cu[i] ? " %d" : "%d", (int)ids[j]);
    printf("\n");
  }
  futon_tokenizer_destroy(tok);
  free(ids);
  free(cu);
  free(off);
  free(text);
  return 0;
}
