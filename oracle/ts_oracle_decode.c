/*
 * ts_oracle_decode.c — CPU restatement of textsift's span decoding: the
 * BIOES Viterbi decoder and the tag-run → span logic.
 *
 * TEST INFRASTRUCTURE ONLY (see ts_oracle.h): the parity checker for the
 * CUDA Viterbi kernel and for "emitted spans byte-identical".
 *
 * Reference (paths relative to packages/textsift/src/):
 *   browser/inference/viterbi.ts:75-145   ViterbiDecoder.decode
 *   browser/inference/viterbi.ts:155-213  buildTransitionMatrix
 *   browser/inference/viterbi.ts:215-225  buildStartScores
 *   browser/inference/spans.ts:29-104     bioesToSpans (token-level runs)
 *
 * Arithmetic as the TypeScript runs it: alpha lives in a Float32Array, so
 * every stored score is rounded to f32; the candidate sums
 * alpha[i] + trans[i] and best + emission are JavaScript doubles; the
 * comparison is a strict '>' starting from -1e30, so the lowest index wins a
 * tie.  The transition and start tables are Float32Arrays filled with -1e30
 * (rounded to f32) except for the allowed entries.
 */
#include <stdint.h>
#include <string.h>

#include "ts_oracle.h"

#define C_TAGS 33
#define N_LABELS 8

static const double kNegInf = -1e30; /* viterbi.ts NEG_INF, a JS double */

/* viterbi.ts:155-225.  trans[to * 33 + from]; cal = {background_stay,
 * background_to_start, inside_to_continue, inside_to_end, end_to_background,
 * end_to_start} (calibration.ts:29-36). */
void tso_viterbi_tables(const float cal[6], float* trans, float* start) {
  const float neg = (float)kNegInf;
  for (int i = 0; i < C_TAGS * C_TAGS; i++) trans[i] = neg;
#define ALLOW(from, to, score) trans[(to) * C_TAGS + (from)] = (score)
  ALLOW(0, 0, cal[0]);
  for (int l = 0; l < N_LABELS; l++) {
    const int B = 1 + 4 * l, I = B + 1, E = B + 2, S = B + 3;
    ALLOW(0, B, cal[1]);
    ALLOW(0, S, cal[1]);
    ALLOW(B, I, cal[2]);
    ALLOW(B, E, cal[3]);
    ALLOW(I, I, cal[2]);
    ALLOW(I, E, cal[3]);
    ALLOW(E, 0, cal[4]);
    ALLOW(S, 0, cal[4]);
    for (int l2 = 0; l2 < N_LABELS; l2++) {
      const int B2 = 1 + 4 * l2, S2 = B2 + 3;
      ALLOW(E, B2, cal[5]);
      ALLOW(E, S2, cal[5]);
      ALLOW(S, B2, cal[5]);
      ALLOW(S, S2, cal[5]);
    }
  }
#undef ALLOW
  for (int j = 0; j < C_TAGS; j++) start[j] = neg;
  start[0] = 0.0f;
  for (int l = 0; l < N_LABELS; l++) {
    start[1 + 4 * l] = 0.0f;
    start[4 + 4 * l] = 0.0f;
  }
}

/* viterbi.ts:75-145.  logits f32[T][33]; alpha f32 and back u8 scratch of
 * T * 33 entries each are supplied by the caller. */
void tso_viterbi(const float* logits, uint32_t T, const float cal[6], uint8_t* tags, float* alpha,
                 uint8_t* back) {
  if (T == 0) return;
  float trans[C_TAGS * C_TAGS], start[C_TAGS];
  tso_viterbi_tables(cal, trans, start);
  for (int j = 0; j < C_TAGS; j++) {
    alpha[j] = (float)((double)start[j] + (double)logits[j]);
    back[j] = 0xFF;
  }
  for (uint32_t t = 1; t < T; t++) {
    const float* prev = alpha + (size_t)(t - 1) * C_TAGS;
    float* cur = alpha + (size_t)t * C_TAGS;
    for (int j = 0; j < C_TAGS; j++) {
      double best = kNegInf;
      int arg = 0;
      const float* col = trans + j * C_TAGS;
      for (int i = 0; i < C_TAGS; i++) {
        const double s = (double)prev[i] + (double)col[i];
        if (s > best) {
          best = s;
          arg = i;
        }
      }
      cur[j] = (float)(best + (double)logits[(size_t)t * C_TAGS + j]);
      back[(size_t)t * C_TAGS + j] = (uint8_t)arg;
    }
  }
  const float* last = alpha + (size_t)(T - 1) * C_TAGS;
  double best_final = kNegInf;
  int final_tag = 0;
  for (int j = 0; j < C_TAGS; j++) {
    if ((double)last[j] > best_final) {
      best_final = (double)last[j];
      final_tag = j;
    }
  }
  tags[T - 1] = (uint8_t)final_tag;
  for (uint32_t t = T - 1; t > 0; t--) tags[t - 1] = back[(size_t)t * C_TAGS + tags[t]];
}

/* spans.ts:29-104, token level: each emitted span is {first token, last
 * token, label}.  (The character mapping and whitespace trim of emit(),
 * spans.ts:106-140, run on the host over the tokenizer's offsets.) */
static void emit(int32_t* out, uint32_t cap, uint32_t* n, int32_t a, int32_t b, int32_t label) {
  if (*n < cap) {
    out[3 * *n + 0] = a;
    out[3 * *n + 1] = b;
    out[3 * *n + 2] = label;
  }
  (*n)++;
}

uint32_t tso_bioes_spans(const uint8_t* tags, uint32_t T, int32_t* out, uint32_t cap) {
  uint32_t n = 0;
  int open_label = -1, open_start = 0;
  for (uint32_t t = 0; t < T; t++) {
    const int tag = tags[t];
    if (tag == 0) { /* O */
      if (open_label >= 0) {
        emit(out, cap, &n, open_start, (int32_t)t - 1, open_label);
        open_label = -1;
      }
      continue;
    }
    const int label = (tag - 1) / 4, boundary = (tag - 1) % 4; /* describeTag: B I E S */
    if (boundary == 3) { /* S */
      if (open_label >= 0) {
        emit(out, cap, &n, open_start, (int32_t)t - 1, open_label);
        open_label = -1;
      }
      emit(out, cap, &n, (int32_t)t, (int32_t)t, label);
    } else if (boundary == 2) { /* E */
      if (open_label >= 0 && open_label == label) {
        emit(out, cap, &n, open_start, (int32_t)t, label);
        open_label = -1;
      } else {
        if (open_label >= 0) {
          emit(out, cap, &n, open_start, (int32_t)t - 1, open_label);
          open_label = -1;
        }
        emit(out, cap, &n, (int32_t)t, (int32_t)t, label);
      }
    } else if (boundary == 1) { /* I */
      if (open_label < 0 || open_label != label) {
        if (open_label >= 0) emit(out, cap, &n, open_start, (int32_t)t - 1, open_label);
        open_label = label;
        open_start = (int)t;
      }
    } else { /* B */
      if (open_label >= 0) emit(out, cap, &n, open_start, (int32_t)t - 1, open_label);
      open_label = label;
      open_start = (int)t;
    }
  }
  if (open_label >= 0) emit(out, cap, &n, open_start, (int32_t)T - 1, open_label);
  return n;
}
