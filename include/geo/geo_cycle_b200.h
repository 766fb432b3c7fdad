/* geo_cycle_b200.h -- the geo_cycle model runner (text model IR, streaming CSV
 * training, text checkpoints, prediction, C export) on libgeo_b200.
 *
 * Replaces the reference's geo_cycle tool: tools/geo_cycle.c (command line),
 * tools/geo_cycle_loader.c:108-310 (model IR "geo_model_ir=8"),
 * tools/geo_cycle_io.c:8-192 (checkpoint "geo_cycle_checkpoint=8", save and
 * load), :194-323 (train), :325-395 (predict), :397-470 (export-c),
 * :472-502 (check), tools/geo_cycle_common.c (line and number grammar).
 * File formats, accepted inputs, printed PASS lines and error messages are the
 * reference's. The model runs on the GPU: stateless models without a reset
 * column train each minibatch of `batch_size` rows in one batched call
 * (geo_b200_v8_batch_train_step semantics, rows uploaded to the device once
 * per run) and predict in one batched forward; models with STATE nodes or a
 * reset column run the per-row geo_v8_* loop of the reference (the rows depend
 * on one another through the states).
 *
 * All functions return 1 on success and 0 on failure (messages on stderr),
 * like the reference's geo_cycle_* functions. */
#ifndef GEO_CYCLE_B200_H
#define GEO_CYCLE_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct geo_b200_cycle_model geo_b200_cycle_model_t;

/* Loads a model IR file; *model is NULL on failure. */
int geo_b200_cycle_load_model(const char *path, geo_b200_cycle_model_t **model);
void geo_b200_cycle_free(geo_b200_cycle_model_t *model);

/* Forward + backward on fixed probe inputs; prints GEO_CYCLE_CHECK: PASS ... */
int geo_b200_cycle_check(geo_b200_cycle_model_t *model);

/* Trains `epochs` epochs over the CSV rows of data_path (optionally resuming
 * from resume_path, which may be NULL) and writes checkpoint_path atomically;
 * prints GEO_CYCLE_TRAIN: PASS ... */
int geo_b200_cycle_train(geo_b200_cycle_model_t *model, const char *data_path, const char *checkpoint_path,
                         const char *resume_path);

/* Writes the output node's value for every CSV row of input_path to
 * output_path (%.17g, comma separated); prints GEO_CYCLE_PREDICT: PASS ... */
int geo_b200_cycle_predict(geo_b200_cycle_model_t *model, const char *input_path, const char *output_path);

/* C header with the trained parameters; prints GEO_CYCLE_EXPORT_C: PASS ... */
int geo_b200_cycle_export_c(geo_b200_cycle_model_t *model, const char *path, const char *symbol);

int geo_b200_cycle_save_checkpoint(const geo_b200_cycle_model_t *model, const char *path);
int geo_b200_cycle_load_checkpoint(geo_b200_cycle_model_t *model, const char *path);

/* The command line of the reference tool (check | train | predict | export-c |
 * --version), plus the model compiler's two commands (compile <model.json>
 * <model.geoir> | validate <model.json>); returns the process exit status. */
int geo_b200_cycle_main(int argc, char **argv);

/* ---- model compiler: JSON model documents -> model IR ------------------------
 * Replaces the reference's tools/geo_model.py (compile / validate): the same
 * accepted documents, rules, rule order and messages, the same IR bytes
 * (including the Mersenne-Twister stream of `random:` initialisers). */

/* Compiles the UTF-8 text of a model document. On success returns 1, sets
 * *ir_text (may be NULL to validate only) to the NUL-terminated IR text
 * (release it with geo_b200_model_free_text) and writes the summary
 * "nodes=.. parameters=.. inputs=.. targets=.. states=.. blade_count=..
 * batch_size=.." into `summary`; on rejection returns 0 and writes the
 * reference compiler's message into `error`. */
int geo_b200_model_compile_text(const char *json_text, size_t json_length, char **ir_text, char *summary,
                                size_t summary_capacity, char *error, size_t error_capacity);
void geo_b200_model_free_text(char *text);

/* Reads model_path, compiles it and writes ir_path atomically (temporary file,
 * fsync, rename), printing "GEO_MODEL_COMPILE: PASS output=<ir_path> <summary>";
 * with ir_path NULL only validates ("GEO_MODEL_VALIDATE: PASS <summary>").
 * Rejections print "geo_model: <message>" on stderr and return 0. */
int geo_b200_model_compile(const char *model_path, const char *ir_path);

#ifdef __cplusplus
}
#endif

#endif
