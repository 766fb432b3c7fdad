// cycle.cpp -- the geo_cycle model runner on libgeo_b200 (geo/geo_cycle_b200.h).
//
// Text formats and command behaviour follow the reference tool
// (tools/geo_cycle_common.c grammar, tools/geo_cycle_loader.c:108-310 model IR,
// tools/geo_cycle_io.c checkpoint/train/predict/export-c/check). Training of a
// stateless model without a reset column runs each minibatch as one batched
// GPU call (v8::run_batch) followed by the program's optimizer step; stateful
// models run the reference's per-row loop through the geo_v8_* runtime.
#include <cuda_runtime.h>
#include <ctype.h>
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "geo/full_cycle_v8.h"
#include "geo/geo_cycle_b200.h"
#include "v8_internal.h"

#define GEO_CYCLE_VERSION "8.0"

struct geo_b200_cycle_model {
    geo_v8_program_t program;
    bool program_live = false;
    geo_v8_optimizer_t optimizer = GEO_V8_OPTIMIZER_ADAM;
    double learning_rate = 0.01, beta1 = 0.9, beta2 = 0.999, epsilon = 1e-8;
    size_t epochs = 1, batch_size = 1;
    int reset_state_each_epoch = 1, reset_column = 0;
    geo_v8_node_id_t output_node = GEO_V8_INVALID_NODE;
    std::vector<geo_v8_node_id_t> inputs, targets, parameters, states;
    std::vector<geo_operator_mv_f64_t> initial_states;
};

namespace {

// ---------------------------------------------------------------- text grammar

std::string trim(const std::string &s) {
    size_t a = 0, b = s.size();
    while (a < b && isspace((unsigned char)s[a])) ++a;
    while (b > a && isspace((unsigned char)s[b - 1])) --b;
    return s.substr(a, b - a);
}

bool rest_blank(const char *p) {
    while (*p != '\0' && isspace((unsigned char)*p)) ++p;
    return *p == '\0';
}

// Reads one '\n'-terminated line (the terminator is dropped); false at end of file.
bool read_line(FILE *f, std::string &line) {
    line.clear();
    int ch;
    bool any = false;
    while ((ch = fgetc(f)) != EOF) {
        any = true;
        if (ch == '\n') return true;
        line.push_back((char)ch);
    }
    return any && !line.empty();
}

bool parse_size(const std::string &t, size_t *out) {
    const char *s = t.c_str();
    char *end = nullptr;
    errno = 0;
    const unsigned long long v = strtoull(s, &end, 10);
    if (errno != 0 || end == s || !rest_blank(end) || v > (unsigned long long)SIZE_MAX) return false;
    *out = (size_t)v;
    return true;
}

bool parse_u64(const std::string &t, uint64_t *out) {
    const char *s = t.c_str();
    char *end = nullptr;
    errno = 0;
    const unsigned long long v = strtoull(s, &end, 10);
    if (errno != 0 || end == s || !rest_blank(end)) return false;
    *out = (uint64_t)v;
    return true;
}

bool parse_double(const std::string &t, double *out) {
    const char *s = t.c_str();
    char *end = nullptr;
    errno = 0;
    const double v = strtod(s, &end);
    if (errno != 0 || end == s || !rest_blank(end) || !isfinite(v)) return false;
    *out = v;
    return true;
}

bool parse_bool(const std::string &t, int *out) {
    if (t == "0") { *out = 0; return true; }
    if (t == "1") { *out = 1; return true; }
    return false;
}

// Comma-separated fields with empty fields skipped (the reference splits with strtok).
std::vector<std::string> split_fields(const std::string &t) {
    std::vector<std::string> out;
    size_t i = 0;
    while (i <= t.size()) {
        const size_t j = t.find(',', i);
        const std::string piece = t.substr(i, j == std::string::npos ? std::string::npos : j - i);
        if (!piece.empty()) out.push_back(trim(piece));
        if (j == std::string::npos) break;
        i = j + 1;
    }
    return out;
}

bool parse_signature(const std::string &t, uint8_t dimension, int8_t *sig) {
    if (t.size() >= 128) return false;
    const std::vector<std::string> f = split_fields(t);
    if (f.size() != dimension) return false;
    for (size_t i = 0; i < f.size(); ++i) {
        const char *s = f[i].c_str();
        char *end = nullptr;
        errno = 0;
        const long v = strtol(s, &end, 10);
        if (errno != 0 || end == s || !rest_blank(end) || (v != 1 && v != -1)) return false;
        sig[i] = (int8_t)v;
    }
    return true;
}

// Numbers separated by commas (optional blanks, a trailing comma allowed);
// with `row` set, '#' ends the list (CSV rows may carry comments).
bool parse_numbers(const char *cursor, double *out, size_t count, bool row) {
    size_t n = 0;
    while (*cursor != '\0') {
        while (*cursor != '\0' && isspace((unsigned char)*cursor)) ++cursor;
        if (row && (*cursor == '\0' || *cursor == '#')) break;
        char *end = nullptr;
        errno = 0;
        const double v = strtod(cursor, &end);
        if (errno != 0 || end == cursor || !isfinite(v) || n >= count) return false;
        out[n++] = v;
        cursor = end;
        while (*cursor != '\0' && isspace((unsigned char)*cursor)) ++cursor;
        if (*cursor == ',') ++cursor;
        else if (*cursor != '\0' && !(row && *cursor == '#')) return false;
    }
    return n == count;
}

void mv_init(geo_operator_mv_f64_t *v, uint8_t dimension, const int8_t *sig) {
    memset(v, 0, sizeof(*v));
    v->dimension = dimension;
    memcpy(v->signature, sig, dimension);
}

// "key=value" with both sides trimmed; false when there is no '='.
bool key_value(const std::string &raw, std::string &key, std::string &value) {
    const size_t eq = raw.find('=');
    if (eq == std::string::npos) return false;
    key = trim(raw.substr(0, eq));
    value = trim(raw.substr(eq + 1));
    return true;
}

// Writes to <path>.tmp and renames it over `path` when complete.
struct AtomicFile {
    std::string path, temporary;
    FILE *f = nullptr;
    bool open(const char *p) {
        path = p;
        temporary = path + ".tmp";
        if (temporary.size() >= 1024) return false;
        f = fopen(temporary.c_str(), "wb");
        return f != nullptr;
    }
    bool finish() {
        const bool ok = fflush(f) == 0;
        const bool closed = fclose(f) == 0;
        f = nullptr;
        if (!ok || !closed) {
            remove(temporary.c_str());
            return false;
        }
        remove(path.c_str());
        if (rename(temporary.c_str(), path.c_str()) != 0) {
            remove(temporary.c_str());
            return false;
        }
        return true;
    }
    void abandon() {
        if (f) fclose(f);
        f = nullptr;
        remove(temporary.c_str());
    }
};

void write_vector(FILE *f, const double *v, size_t n) {
    for (size_t i = 0; i < n; ++i) fprintf(f, "%s%.17g", i == 0 ? "" : ",", v[i]);
}

size_t blades_of(const geo_b200_cycle_model_t *m) { return (size_t)1u << m->program.dimension; }

bool reset_states(geo_b200_cycle_model_t *m) {
    for (size_t i = 0; i < m->states.size(); ++i)
        if (geo_v8_set_value(&m->program, m->states[i], &m->initial_states[i]) != GEO_V8_OK) return false;
    return true;
}

bool set_leaves(geo_b200_cycle_model_t *m, const std::vector<geo_v8_node_id_t> &nodes, const double *values) {
    const size_t nb = blades_of(m);
    for (size_t i = 0; i < nodes.size(); ++i) {
        geo_operator_mv_f64_t v = m->program.nodes[nodes[i]].value;
        memcpy(v.coefficients, values + i * nb, nb * sizeof(double));
        if (geo_v8_set_value(&m->program, nodes[i], &v) != GEO_V8_OK) return false;
    }
    return true;
}

// All data rows of a CSV file (blank and '#' lines skipped): 1 read, 0 bad row, -1 cannot open.
int read_rows(const char *path, size_t expected, std::vector<double> &rows, size_t *count) {
    FILE *f = fopen(path, "rb");
    if (f == nullptr) return -1;
    std::string line;
    std::vector<double> row(expected ? expected : 1);
    *count = 0;
    bool ok = true;
    while (read_line(f, line)) {
        const std::string t = trim(line);
        if (t.empty() || t[0] == '#') continue;
        if (!parse_numbers(t.c_str(), row.data(), expected, true)) {
            ok = false;
            break;
        }
        rows.insert(rows.end(), row.begin(), row.begin() + (ptrdiff_t)expected);
        ++*count;
    }
    if (ferror(f)) ok = false;
    fclose(f);
    return ok ? 1 : 0;
}

bool stateless(const geo_b200_cycle_model_t *m) { return m->states.empty() && !m->reset_column; }

// Device copy of host rows (freed by the destructor).
struct DeviceRows {
    double *ptr = nullptr;
    ~DeviceRows() {
        if (ptr) cudaFree(ptr);
    }
    bool upload(const std::vector<double> &rows) {
        if (cudaMalloc((void **)&ptr, rows.size() * sizeof(double)) != cudaSuccess) {
            (void)cudaGetLastError();
            ptr = nullptr;
            return false;
        }
        return cudaMemcpy(ptr, rows.data(), rows.size() * sizeof(double), cudaMemcpyHostToDevice) == cudaSuccess;
    }
};

// One minibatch of rows through the batched path, then the program's optimizer step.
bool batched_step(geo_b200_cycle_model_t *m, const double *device_rows, size_t row_doubles, size_t count,
                  double *loss_sum) {
    geo_v8_program_t *p = &m->program;
    const size_t nb = blades_of(m);
    std::vector<geo::v8::RowLeaf> leaves;
    size_t column = (size_t)m->reset_column;
    for (geo_v8_node_id_t id : m->inputs) {
        leaves.push_back({id, 1, column});
        column += nb;
    }
    for (geo_v8_node_id_t id : m->targets) {
        leaves.push_back({id, 1, column});
        column += nb;
    }
    (void)geo_v8_zero_grad(p);
    std::vector<double> grads;
    if (geo::v8::run_batch(p, leaves, {device_rows, row_doubles}, {nullptr, 0}, GEO_V8_INVALID_NODE, nullptr, count,
                           1, loss_sum, &grads) != GEO_V8_OK)
        return false;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (geo::v8::leaf_kind(p->nodes[i].kind) && p->nodes[i].requires_grad)
            memcpy(p->nodes[i].gradient.coefficients, &grads[(size_t)i * 64], nb * sizeof(double));
    p->gradient_samples = count;
    p->forward_valid = 1u;
    p->backward_valid = 1u;
    return geo_v8_optimizer_step(p, m->optimizer, m->learning_rate, m->beta1, m->beta2, m->epsilon,
                                 1.0 / (double)count) == GEO_V8_OK;
}

}  // namespace

// ------------------------------------------------------------------ model IR

extern "C" void geo_b200_cycle_free(geo_b200_cycle_model_t *m) {
    if (m == nullptr) return;
    if (m->program_live) geo_v8_program_free(&m->program);
    delete m;
}

extern "C" int geo_b200_cycle_load_model(const char *path, geo_b200_cycle_model_t **out) {
    if (out == nullptr) return 0;
    *out = nullptr;
    FILE *f = path ? fopen(path, "rb") : nullptr;
    if (f == nullptr) {
        fprintf(stderr, "geo_cycle: cannot open model '%s'\n", path ? path : "");
        return 0;
    }
    geo_b200_cycle_model_t *m = new geo_b200_cycle_model_t();
    memset(&m->program, 0, sizeof(m->program));
    uint8_t dimension = 0;
    int8_t signature[6] = {0};
    size_t node_count = 0, nodes_read = 0;
    geo_v8_node_id_t loss = GEO_V8_INVALID_NODE, output = GEO_V8_INVALID_NODE;
    bool header = false, dim_seen = false, sig_seen = false, opt_seen = false, count_seen = false;
    bool loss_seen = false, out_seen = false, end_seen = false, ok = true;
    std::string line, key, value;
    while (ok && read_line(f, line)) {
        const std::string t = trim(line);
        if (t.empty() || t[0] == '#') continue;
        if (!key_value(t, key, value)) { ok = false; break; }
        if (key == "geo_model_ir") {
            ok = value == "8" && !header;
            header = true;
        } else if (key == "dimension") {
            size_t v;
            ok = parse_size(value, &v) && v >= 1 && v <= 6 && !dim_seen;
            dimension = (uint8_t)v;
            dim_seen = true;
        } else if (key == "signature") {
            ok = dim_seen && !sig_seen && parse_signature(value, dimension, signature);
            sig_seen = true;
        } else if (key == "optimizer") {
            size_t v;
            ok = parse_size(value, &v) && (v == 1 || v == 2) && !opt_seen;
            m->optimizer = (geo_v8_optimizer_t)v;
            opt_seen = true;
        } else if (key == "learning_rate") {
            ok = parse_double(value, &m->learning_rate) && m->learning_rate > 0.0;
        } else if (key == "beta1") {
            ok = parse_double(value, &m->beta1) && m->beta1 >= 0.0 && m->beta1 < 1.0;
        } else if (key == "beta2") {
            ok = parse_double(value, &m->beta2) && m->beta2 >= 0.0 && m->beta2 < 1.0;
        } else if (key == "epsilon") {
            ok = parse_double(value, &m->epsilon) && m->epsilon > 0.0;
        } else if (key == "epochs") {
            ok = parse_size(value, &m->epochs) && m->epochs != 0;
        } else if (key == "batch_size") {
            ok = parse_size(value, &m->batch_size) && m->batch_size != 0;
        } else if (key == "reset_state_each_epoch") {
            ok = parse_bool(value, &m->reset_state_each_epoch);
        } else if (key == "reset_column") {
            ok = parse_bool(value, &m->reset_column);
        } else if (key == "node_count") {
            ok = header && sig_seen && opt_seen && !count_seen && parse_size(value, &node_count) && node_count != 0 &&
                 node_count <= (size_t)UINT32_MAX &&
                 geo_v8_program_init(&m->program, dimension, signature, GEO_V8_PAIRING_COEFFICIENT_EUCLIDEAN,
                                     node_count) == GEO_V8_OK;
            if (ok) m->program_live = true;
            count_seen = true;
        } else if (key == "loss" || key == "output") {
            size_t v;
            bool &seen = key == "loss" ? loss_seen : out_seen;
            ok = parse_size(value, &v) && v <= (size_t)UINT32_MAX && !seen;
            (key == "loss" ? loss : output) = (geo_v8_node_id_t)v;
            seen = true;
        } else if (key == "node") {
            // index,kind,name,left,right,scalar,grade,constraint,requires_grad then a value= line
            const std::vector<std::string> fld = split_fields(value);
            size_t index = 0, kind = 0, left = 0, right = 0, grade = 0, constraint = 0, rg = 0;
            double scalar = 0.0;
            ok = count_seen && nodes_read < node_count && fld.size() == 9 && parse_size(fld[0], &index) &&
                 parse_size(fld[1], &kind) && kind <= 255 && fld[2].size() < GEO_V8_NAME_MAX &&
                 parse_size(fld[3], &left) && left <= UINT32_MAX && parse_size(fld[4], &right) &&
                 right <= UINT32_MAX && parse_double(fld[5], &scalar) && parse_size(fld[6], &grade) &&
                 grade <= 255 && parse_size(fld[7], &constraint) && constraint <= 255 && parse_size(fld[8], &rg) &&
                 rg <= 1 && index == nodes_read && kind >= 1 && kind <= 17 && constraint <= 3;
            std::string vkey, vval;
            ok = ok && read_line(f, line) && key_value(trim(line), vkey, vval) && vkey == "value";
            geo_operator_mv_f64_t initial;
            mv_init(&initial, dimension, signature);
            ok = ok && parse_numbers(vval.c_str(), initial.coefficients, (size_t)1u << dimension, false);
            if (!ok) break;
            geo_v8_node_id_t created = GEO_V8_INVALID_NODE;
            const int k = (int)kind;
            if (k >= GEO_V8_NODE_INPUT && k <= GEO_V8_NODE_STATE) {
                ok = geo_v8_add_leaf(&m->program, (geo_v8_node_kind_t)k, fld[2].c_str(), &initial, (int)rg,
                                     (geo_v8_constraint_t)constraint, &created) == GEO_V8_OK;
            } else if (k == GEO_V8_NODE_ADD || k == GEO_V8_NODE_GEOMETRIC_PRODUCT || k == GEO_V8_NODE_HADAMARD) {
                ok = left < nodes_read && right < nodes_read &&
                     geo_v8_add_binary(&m->program, (geo_v8_node_kind_t)k, fld[2].c_str(), (geo_v8_node_id_t)left,
                                       (geo_v8_node_id_t)right, &created) == GEO_V8_OK;
            } else {
                ok = left < nodes_read && right == GEO_V8_INVALID_NODE &&
                     geo_v8_add_unary(&m->program, (geo_v8_node_kind_t)k, fld[2].c_str(), (geo_v8_node_id_t)left,
                                      scalar, (uint8_t)grade, &created) == GEO_V8_OK;
            }
            ok = ok && (size_t)created == index;
            ++nodes_read;
        } else if (key == "state_update") {
            const size_t comma = value.find(',');
            size_t a = 0, b = 0;
            ok = comma != std::string::npos && parse_size(trim(value.substr(0, comma)), &a) && a <= UINT32_MAX &&
                 parse_size(trim(value.substr(comma + 1)), &b) && b <= UINT32_MAX &&
                 geo_v8_bind_state_update(&m->program, (geo_v8_node_id_t)a, (geo_v8_node_id_t)b) == GEO_V8_OK;
        } else if (key == "end") {
            ok = value == "1" && !end_seen;
            end_seen = true;
        } else {
            ok = false;
        }
    }
    ok = ok && !ferror(f) && header && dim_seen && sig_seen && count_seen && loss_seen && out_seen && end_seen &&
         nodes_read == node_count && loss < node_count && output < node_count &&
         geo_v8_compile(&m->program, loss) == GEO_V8_OK;
    fclose(f);
    if (!ok) {
        fprintf(stderr, "geo_cycle: invalid model IR '%s'\n", path);
        geo_b200_cycle_free(m);
        return 0;
    }
    m->output_node = output;
    for (geo_v8_node_id_t i = 0; i < m->program.node_count; ++i) {
        const int k = m->program.nodes[i].kind;
        if (k == GEO_V8_NODE_INPUT) m->inputs.push_back(i);
        else if (k == GEO_V8_NODE_TARGET) m->targets.push_back(i);
        else if (k == GEO_V8_NODE_PARAMETER) m->parameters.push_back(i);
        else if (k == GEO_V8_NODE_STATE) {
            m->states.push_back(i);
            m->initial_states.push_back(m->program.nodes[i].value);
        }
    }
    if (m->inputs.empty()) {
        geo_b200_cycle_free(m);
        return 0;
    }
    *out = m;
    return 1;
}

// ----------------------------------------------------------------- checkpoint

extern "C" int geo_b200_cycle_save_checkpoint(const geo_b200_cycle_model_t *m, const char *path) {
    if (m == nullptr || path == nullptr) return 0;
    AtomicFile af;
    if (!af.open(path)) return 0;
    FILE *f = af.f;
    const size_t nb = blades_of(m);
    fprintf(f, "geo_cycle_checkpoint=8\n");
    fprintf(f, "dimension=%u\n", (unsigned)m->program.dimension);
    fprintf(f, "signature=");
    for (unsigned i = 0; i < m->program.dimension; ++i) fprintf(f, "%s%d", i == 0 ? "" : ",", (int)m->program.signature[i]);
    fprintf(f, "\noptimizer_step=%llu\n", (unsigned long long)m->program.optimizer_step);
    for (geo_v8_node_id_t id : m->parameters) {
        const geo_v8_node_t *node = &m->program.nodes[id];
        fprintf(f, "parameter=%s,%u\nvalue=", node->name, (unsigned)node->constraint);
        write_vector(f, node->value.coefficients, nb);
        fprintf(f, "\nfirst=");
        write_vector(f, node->first_moment, nb);
        fprintf(f, "\nsecond=");
        write_vector(f, node->second_moment, nb);
        fprintf(f, "\nend_parameter=1\n");
    }
    for (geo_v8_node_id_t id : m->states) {
        const geo_v8_node_t *node = &m->program.nodes[id];
        fprintf(f, "state=%s\nvalue=", node->name);
        write_vector(f, node->value.coefficients, nb);
        fprintf(f, "\nend_state=1\n");
    }
    fprintf(f, "end=1\n");
    return af.finish() ? 1 : 0;
}

extern "C" int geo_b200_cycle_load_checkpoint(geo_b200_cycle_model_t *m, const char *path) {
    if (m == nullptr || path == nullptr) return 0;
    FILE *f = fopen(path, "rb");
    if (f == nullptr) return 0;
    const size_t nb = blades_of(m);
    std::vector<char> pseen(m->parameters.size(), 0), sseen(m->states.size(), 0);
    bool header = false, dim = false, sig = false, step = false, ok = true;
    size_t params = 0, states = 0;
    std::string line, key, value;
    auto position = [](const std::vector<geo_v8_node_id_t> &ids, geo_v8_node_id_t id) -> size_t {
        for (size_t i = 0; i < ids.size(); ++i)
            if (ids[i] == id) return i;
        return SIZE_MAX;
    };
    // The next line must start with "<tag>=" (no blank before '='), followed by the vector.
    auto tagged = [&](const char *tag, double *dst) {
        if (!read_line(f, line)) return false;
        const std::string t = trim(line);
        const std::string prefix = std::string(tag) + "=";
        return t.compare(0, prefix.size(), prefix) == 0 && parse_numbers(t.c_str() + prefix.size(), dst, nb, false);
    };
    while (ok && read_line(f, line)) {
        const std::string t = trim(line);
        if (t.empty() || t[0] == '#') continue;
        if (!key_value(t, key, value)) { ok = false; break; }
        if (key == "geo_cycle_checkpoint") {
            ok = value == "8" && !header;
            header = true;
        } else if (key == "dimension") {
            size_t v;
            ok = parse_size(value, &v) && v == m->program.dimension;
            dim = true;
        } else if (key == "signature") {
            int8_t s[6] = {0};
            ok = parse_signature(value, m->program.dimension, s) &&
                 memcmp(s, m->program.signature, m->program.dimension) == 0;
            sig = true;
        } else if (key == "optimizer_step") {
            ok = parse_u64(value, &m->program.optimizer_step);
            step = true;
        } else if (key == "parameter") {
            const size_t comma = value.find(',');
            size_t constraint = 0;
            ok = comma != std::string::npos && parse_size(trim(value.substr(comma + 1)), &constraint) &&
                 constraint <= 3;
            if (!ok) break;
            const std::string name = trim(value.substr(0, comma));
            const geo_v8_node_id_t id = geo_v8_find_node(&m->program, name.c_str());
            const size_t pos = position(m->parameters, id);
            ok = id != GEO_V8_INVALID_NODE && m->program.nodes[id].kind == GEO_V8_NODE_PARAMETER &&
                 m->program.nodes[id].constraint == (uint8_t)constraint && pos != SIZE_MAX && !pseen[pos];
            if (!ok) break;
            pseen[pos] = 1;
            geo_v8_node_t *node = &m->program.nodes[id];
            ok = tagged("value", node->value.coefficients) && tagged("first", node->first_moment) &&
                 tagged("second", node->second_moment) && read_line(f, line) && trim(line) == "end_parameter=1";
            ++params;
        } else if (key == "state") {
            const geo_v8_node_id_t id = geo_v8_find_node(&m->program, value.c_str());
            const size_t pos = position(m->states, id);
            ok = id != GEO_V8_INVALID_NODE && m->program.nodes[id].kind == GEO_V8_NODE_STATE && pos != SIZE_MAX &&
                 !sseen[pos];
            if (!ok) break;
            sseen[pos] = 1;
            ok = tagged("value", m->program.nodes[id].value.coefficients) && read_line(f, line) &&
                 trim(line) == "end_state=1";
            ++states;
        } else if (key == "end") {
            ok = value == "1";
        } else {
            ok = false;
        }
    }
    ok = ok && !ferror(f) && header && dim && sig && step && params == m->parameters.size() &&
         states == m->states.size();
    fclose(f);
    if (!ok) {
        fprintf(stderr, "geo_cycle: invalid or mismatched checkpoint '%s'\n", path);
        return 0;
    }
    m->program.forward_valid = 0u;
    m->program.backward_valid = 0u;
    m->program.gradient_samples = 0u;
    return 1;
}

// -------------------------------------------------------------------- train

extern "C" int geo_b200_cycle_train(geo_b200_cycle_model_t *m, const char *data_path, const char *checkpoint_path,
                                    const char *resume_path) {
    if (m == nullptr || data_path == nullptr || checkpoint_path == nullptr) return 0;
    const size_t nb = blades_of(m);
    const size_t expected = (size_t)m->reset_column + (m->inputs.size() + m->targets.size()) * nb;
    if (m->targets.empty() || m->parameters.empty()) return 0;
    if (resume_path != nullptr && !geo_b200_cycle_load_checkpoint(m, resume_path)) return 0;
    std::vector<double> rows;
    size_t row_count = 0;
    const int read = read_rows(data_path, expected, rows, &row_count);
    if (read < 0) return 0;  // like the reference: an unreadable data file fails without a message
    bool ok = read == 1 && row_count != 0;
    double initial_loss = NAN, final_loss = NAN;
    uint64_t rows_total = 0;
    DeviceRows device;
    const bool batched = stateless(m);
    if (ok && batched) ok = device.upload(rows);
    for (size_t epoch = 0; ok && epoch < m->epochs; ++epoch) {
        double epoch_loss = 0.0;
        if (m->reset_state_each_epoch && !reset_states(m)) { ok = false; break; }
        if (geo_v8_zero_grad(&m->program) != GEO_V8_OK) { ok = false; break; }
        if (batched) {
            for (size_t first = 0; ok && first < row_count; first += m->batch_size) {
                const size_t count = row_count - first < m->batch_size ? row_count - first : m->batch_size;
                double loss = 0.0;
                ok = batched_step(m, device.ptr + first * expected, expected, count, &loss);
                epoch_loss += loss;
                rows_total += count;
            }
        } else {
            // reference tools/geo_cycle_io.c:222-282, row by row
            size_t batch_count = 0;
            for (size_t r = 0; ok && r < row_count; ++r) {
                const double *v = rows.data() + r * expected;
                size_t offset = 0;
                if (m->reset_column) {
                    if (v[0] != 0.0 && v[0] != 1.0) { ok = false; break; }
                    if (v[0] == 1.0 && !reset_states(m)) { ok = false; break; }
                    offset = 1;
                }
                ok = set_leaves(m, m->inputs, v + offset) && set_leaves(m, m->targets, v + offset + m->inputs.size() * nb) &&
                     geo_v8_forward(&m->program) == GEO_V8_OK;
                if (!ok) break;
                const geo_operator_mv_f64_t *lv = geo_v8_value(&m->program, m->program.loss_node);
                if (lv == nullptr || !isfinite(lv->coefficients[0])) { ok = false; break; }
                epoch_loss += lv->coefficients[0];
                ok = geo_v8_backward(&m->program, batch_count != 0) == GEO_V8_OK &&
                     (m->states.empty() || geo_v8_commit_states(&m->program) == GEO_V8_OK);
                if (!ok) break;
                ++batch_count;
                ++rows_total;
                if (batch_count == m->batch_size) {
                    ok = geo_v8_optimizer_step(&m->program, m->optimizer, m->learning_rate, m->beta1, m->beta2,
                                               m->epsilon, 1.0 / (double)batch_count) == GEO_V8_OK;
                    batch_count = 0;
                }
            }
            if (ok && batch_count != 0)
                ok = geo_v8_optimizer_step(&m->program, m->optimizer, m->learning_rate, m->beta1, m->beta2,
                                           m->epsilon, 1.0 / (double)batch_count) == GEO_V8_OK;
        }
        if (!ok) break;
        epoch_loss /= (double)row_count;
        if (epoch == 0) initial_loss = epoch_loss;
        final_loss = epoch_loss;
    }
    if (!ok) {
        fprintf(stderr, "geo_cycle: invalid training data or runtime failure\n");
        return 0;
    }
    if (!geo_b200_cycle_save_checkpoint(m, checkpoint_path)) return 0;
    printf("GEO_CYCLE_TRAIN: PASS epochs=%zu rows=%llu batch_size=%zu parameters=%zu states=%zu initial_loss=%.17g "
           "final_loss=%.17g checkpoint=%s\n",
           m->epochs, (unsigned long long)rows_total, m->batch_size, m->parameters.size(), m->states.size(),
           initial_loss, final_loss, checkpoint_path);
    return 1;
}

// ------------------------------------------------------------------ predict

extern "C" int geo_b200_cycle_predict(geo_b200_cycle_model_t *m, const char *input_path, const char *output_path) {
    if (m == nullptr || input_path == nullptr || output_path == nullptr) return 0;
    const size_t nb = blades_of(m);
    const size_t expected = (size_t)m->reset_column + m->inputs.size() * nb;
    std::vector<double> rows;
    size_t row_count = 0;
    std::vector<double> predictions;
    const int read = read_rows(input_path, expected, rows, &row_count);
    if (read < 0) return 0;  // unreadable input: no message, as the reference
    bool ok = read == 1 && row_count != 0;
    if (ok && stateless(m)) {
        DeviceRows device;
        double *out = nullptr;
        ok = device.upload(rows) && cudaMalloc((void **)&out, row_count * nb * sizeof(double)) == cudaSuccess;
        std::vector<geo::v8::RowLeaf> leaves;
        for (size_t i = 0; i < m->inputs.size(); ++i) leaves.push_back({m->inputs[i], 1, i * nb});
        ok = ok && geo::v8::run_batch(&m->program, leaves, {device.ptr, expected}, {nullptr, 0}, m->output_node, out,
                                      row_count, 0, nullptr, nullptr) == GEO_V8_OK;
        predictions.resize(row_count * nb);
        ok = ok && cudaMemcpy(predictions.data(), out, predictions.size() * sizeof(double), cudaMemcpyDeviceToHost) ==
                       cudaSuccess;
        if (out) cudaFree(out);
        (void)cudaGetLastError();
    } else if (ok) {
        // reference tools/geo_cycle_io.c:347-373, row by row
        for (size_t r = 0; ok && r < row_count; ++r) {
            const double *v = rows.data() + r * expected;
            size_t offset = 0;
            if (m->reset_column) {
                if (v[0] != 0.0 && v[0] != 1.0) { ok = false; break; }
                if (v[0] == 1.0 && !reset_states(m)) { ok = false; break; }
                offset = 1;
            }
            ok = set_leaves(m, m->inputs, v + offset) && geo_v8_forward(&m->program) == GEO_V8_OK;
            const geo_operator_mv_f64_t *pv = ok ? geo_v8_value(&m->program, m->output_node) : nullptr;
            ok = ok && pv != nullptr;
            if (ok) predictions.insert(predictions.end(), pv->coefficients, pv->coefficients + nb);
            ok = ok && (m->states.empty() || geo_v8_commit_states(&m->program) == GEO_V8_OK);
        }
    }
    AtomicFile af;
    if (ok && af.open(output_path)) {
        for (size_t r = 0; r < row_count; ++r) {
            write_vector(af.f, predictions.data() + r * nb, nb);
            fprintf(af.f, "\n");
        }
        if (!af.finish()) return 0;
        printf("GEO_CYCLE_PREDICT: PASS rows=%llu output=%s\n", (unsigned long long)row_count, output_path);
        return 1;
    }
    if (af.f) af.abandon();
    fprintf(stderr, "geo_cycle: invalid prediction input or runtime failure\n");
    return 0;
}

// ---------------------------------------------------------- export-c, check

extern "C" int geo_b200_cycle_export_c(geo_b200_cycle_model_t *m, const char *path, const char *symbol) {
    if (m == nullptr || path == nullptr || symbol == nullptr) return 0;
    if (!(isalpha((unsigned char)symbol[0]) || symbol[0] == '_')) return 0;
    for (const char *c = symbol + 1; *c; ++c)
        if (!(isalnum((unsigned char)*c) || *c == '_')) return 0;
    AtomicFile af;
    if (!af.open(path)) return 0;
    FILE *f = af.f;
    const size_t nb = blades_of(m);
    fprintf(f, "#ifndef %s_GEO_V8_MODEL_H\n#define %s_GEO_V8_MODEL_H\n\n", symbol, symbol);
    fprintf(f, "#include <stddef.h>\n#include <stdint.h>\n\n");
    fprintf(f, "#define %s_DIMENSION %uu\n#define %s_BLADE_COUNT %zuu\n#define %s_PARAMETER_COUNT %zuu\n\n", symbol,
            (unsigned)m->program.dimension, symbol, nb, symbol, m->parameters.size());
    fprintf(f, "static const int8_t %s_signature[%u] = {", symbol, (unsigned)m->program.dimension);
    for (unsigned i = 0; i < m->program.dimension; ++i) fprintf(f, "%s%d", i == 0 ? "" : ", ", (int)m->program.signature[i]);
    fprintf(f, "};\n");
    for (geo_v8_node_id_t id : m->parameters) {
        const geo_v8_node_t *node = &m->program.nodes[id];
        fprintf(f, "static const double %s_%s[%zu] = {\n", symbol, node->name, nb);
        for (size_t b = 0; b < nb; ++b) fprintf(f, "    %.17g%s\n", node->value.coefficients[b], b + 1 == nb ? "" : ",");
        fprintf(f, "};\n");
    }
    fprintf(f, "\n#endif\n");
    if (!af.finish()) return 0;
    printf("GEO_CYCLE_EXPORT_C: PASS parameters=%zu header=%s\n", m->parameters.size(), path);
    return 1;
}

extern "C" int geo_b200_cycle_check(geo_b200_cycle_model_t *m) {
    if (m == nullptr) return 0;
    const size_t nb = blades_of(m);
    for (size_t i = 0; i < m->inputs.size(); ++i) {
        geo_operator_mv_f64_t probe = m->program.nodes[m->inputs[i]].value;
        for (size_t b = 0; b < nb; ++b) probe.coefficients[b] = (double)((int)((b + 1) * (i + 3) % 17) - 8) / 19.0;
        if (geo_v8_set_value(&m->program, m->inputs[i], &probe) != GEO_V8_OK) return 0;
    }
    if (geo_v8_forward(&m->program) != GEO_V8_OK || geo_v8_backward(&m->program, 0) != GEO_V8_OK) return 0;
    printf("GEO_CYCLE_CHECK: PASS nodes=%u parameters=%zu inputs=%zu targets=%zu states=%zu abi=0x%08x "
           "external_autograd=NONE\n",
           (unsigned)m->program.node_count, m->parameters.size(), m->inputs.size(), m->targets.size(),
           m->states.size(), geo_v8_abi_version());
    return 1;
}

// -------------------------------------------------------------- command line

extern "C" int geo_b200_cycle_main(int argc, char **argv) {
    auto usage = [](FILE *s) {
        fprintf(s,
                "geo_cycle %s\nGEO V8 arbitrary-graph full-cycle runner.\n\nCommands:\n"
                "  geo_cycle check <model.geoir>\n"
                "  geo_cycle train <model.geoir> <train.csv> <checkpoint> [resume-checkpoint]\n"
                "  geo_cycle predict <model.geoir> <checkpoint> <input.csv> <output.csv>\n"
                "  geo_cycle export-c <model.geoir> <checkpoint> <header.h> <symbol>\n",
                GEO_CYCLE_VERSION);
    };
    if (argc < 2) {
        usage(stderr);
        return EXIT_FAILURE;
    }
    const std::string cmd = argv[1];
    if (cmd == "--version") {
        printf("geo_cycle %s GEO_V8_ABI=0x%08x\n", GEO_CYCLE_VERSION, geo_v8_abi_version());
        return EXIT_SUCCESS;
    }
    // The model compiler (JSON document -> model IR), beside the runner's commands.
    if (cmd == "compile" && argc == 4) return geo_b200_model_compile(argv[2], argv[3]) ? EXIT_SUCCESS : EXIT_FAILURE;
    if (cmd == "validate" && argc == 3) return geo_b200_model_compile(argv[2], nullptr) ? EXIT_SUCCESS : EXIT_FAILURE;
    geo_b200_cycle_model_t *m = nullptr;
    int success = 0;
    if (cmd == "check" && argc == 3) {
        if (geo_b200_cycle_load_model(argv[2], &m)) success = geo_b200_cycle_check(m);
    } else if (cmd == "train" && (argc == 5 || argc == 6)) {
        if (geo_b200_cycle_load_model(argv[2], &m))
            success = geo_b200_cycle_train(m, argv[3], argv[4], argc == 6 ? argv[5] : nullptr);
    } else if (cmd == "predict" && argc == 6) {
        if (geo_b200_cycle_load_model(argv[2], &m) && geo_b200_cycle_load_checkpoint(m, argv[3]))
            success = geo_b200_cycle_predict(m, argv[4], argv[5]);
    } else if (cmd == "export-c" && argc == 6) {
        if (geo_b200_cycle_load_model(argv[2], &m) && geo_b200_cycle_load_checkpoint(m, argv[3]))
            success = geo_b200_cycle_export_c(m, argv[4], argv[5]);
    } else {
        usage(stderr);
    }
    geo_b200_cycle_free(m);
    return success ? EXIT_SUCCESS : EXIT_FAILURE;
}
