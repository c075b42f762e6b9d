/*
 * futon_tokenizer.h — C ABI of the native WordPiece tokenizer in
 * libfuton_cuda (host code only: no GPU is needed to call it).
 *
 * The text side of futon's native Provider, feeding futon_cuda_encode:
 * futon_tokenizer_encode_batch writes exactly the packed ids and cu_seqlens
 * that futon_cuda_encode / futon_cuda_encode_batch take. Ids are the
 * reference tokenizer's, bit for bit. Plain C types only; every entry point
 * returns 0 or a FUTON_E* code (futon_cuda.h) and writes a UTF-8 message
 * into err[errlen] on failure.
 *
 * Reference interfaces replaced (paths within github.com/bobbyhiddn/futon):
 *   native/tokenizer.go:15-55   TokenizerConfig        -> futon_tokenizer_cfg
 *   native/tokenizer.go:90-136  NewTokenizer           -> futon_tokenizer_create
 *   native/tokenizer.go:138     Tokenizer.VocabSize    -> futon_tokenizer_vocab_size
 *   native/tokenizer.go:141     Tokenizer.PadID        -> futon_tokenizer_pad_id
 *   native/tokenizer.go:143-184 Tokenizer.Encode       -> futon_tokenizer_encode
 *   native/provider.go:152-202  EmbedBatch's per-text Encode calls
 *                                                      -> futon_tokenizer_encode_batch
 */
#ifndef FUTON_TOKENIZER_H
#define FUTON_TOKENIZER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* TokenizerConfig (a pack config's "tokenizer" object). Zero / NULL / ""
 * fields take the reference's defaults (applyDefaults): 100 characters per
 * word, "[CLS]", "[SEP]", "[UNK]", "[PAD]", "[MASK]". */
typedef struct futon_tokenizer_cfg {
  int32_t do_lower_case;            /* lowercase + NFD accent stripping */
  int32_t tokenize_chinese_chars;   /* isolate CJK ideographs */
  int32_t max_input_chars_per_word; /* longer words become [UNK] */
  const char* cls_token;
  const char* sep_token;
  const char* unk_token;
  const char* pad_token;
  const char* mask_token;
} futon_tokenizer_cfg;

typedef struct futon_tokenizer futon_tokenizer;

/* Builds a tokenizer from the bytes of a vocab.txt (one token per line, line
 * number = id; LF or CRLF; a repeated token keeps its last id). Fails like
 * NewTokenizer: an empty vocab, a line over 1 MiB, or a special token that
 * is not in the vocab. The bytes are not retained. The tokenizer is
 * read-only after creation and safe to use from many threads at once. */
int futon_tokenizer_create(const char* vocab, size_t vocab_len, const futon_tokenizer_cfg* cfg,
                           futon_tokenizer** out, char* err, size_t errlen);

void futon_tokenizer_destroy(futon_tokenizer* tok);

/* Number of distinct tokens in the vocab (VocabSize), or -1 for NULL. */
int futon_tokenizer_vocab_size(const futon_tokenizer* tok);

/* Id of the [PAD] token (PadID), or -1 for NULL. */
int futon_tokenizer_pad_id(const futon_tokenizer* tok);

/* Encode: the ids of text[0, len) (UTF-8; invalid bytes are dropped) wrapped
 * in [CLS] … [SEP] and head-truncated to at most max(max_seq_len, 2) ids.
 * Writes *n_ids; fails with FUTON_EINVAL, writing nothing into ids but the
 * needed count into *n_ids, if it exceeds cap. */
int futon_tokenizer_encode(const futon_tokenizer* tok, const char* text, size_t len,
                           int max_seq_len, int32_t* ids, int cap, int* n_ids, char* err,
                           size_t errlen);

/* Encode of ntexts texts at once, on nthreads host threads (0 = every
 * hardware thread). Text i is bytes [text_offsets[i], text_offsets[i+1]) of
 * `text` (offsets non-decreasing, from 0 or more). Writes cu_seqlens[0..
 * ntexts] (cu_seqlens[0] = 0) and the ids of text i into ids[cu_seqlens[i],
 * cu_seqlens[i+1]): the packed layout futon_cuda_encode takes. If the total
 * exceeds ids_cap (ntexts × max(max_seq_len, 2) always suffices) it fails with
 * FUTON_EINVAL after writing cu_seqlens only, so the caller can size ids
 * from cu_seqlens[ntexts] and call again. Results equal futon_tokenizer_encode
 * per text for every thread count. */
int futon_tokenizer_encode_batch(const futon_tokenizer* tok, const char* text,
                                 const int64_t* text_offsets, int ntexts, int max_seq_len,
                                 int nthreads, int32_t* ids, int64_t ids_cap,
                                 int32_t* cu_seqlens, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif /* FUTON_TOKENIZER_H */
