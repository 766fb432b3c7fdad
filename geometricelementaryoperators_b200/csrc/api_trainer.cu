// api_trainer.cu -- resident trainer and NCCL data parallelism (geo/geo_b200.h).
//
// The trainer batches the reference V8 full-cycle loop for the graph
// x*w -> add(., scale(t, -1)) -> squared_norm (reference
// benchmarks/bench_v8_full_cycle.c:35-56 builds exactly this graph; the
// per-sample loop is tools/geo_cycle_io.c:194-323): one fused streaming pass
// per minibatch computes the summed parameter gradient and loss, then one tiny
// kernel applies geo_v8_optimizer_step's SGD/Adam update
// (reference src/full_cycle_v8.c:942-1041) on the device. The Adam bias terms
// 1 - beta^t are computed on the host with libm pow, as the reference does.
//
// Data parallelism: each rank reduces its CTA records into one rank record
// (2^n gradient sums, loss, probes), the records are all-gathered over NCCL
// (a 576-byte message) and every rank sums them in rank order before the
// identical update, so replicas stay bit-identical without a broadcast.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>  // types and NCCL_CONFIG_INITIALIZER only; entry points are resolved at run time
#include <string.h>

#include <chrono>
#include <new>
#include <thread>

#include "geo/geo_b200.h"
#include "geo_runtime.h"
#include "representation.h"

struct geo_b200_comm {
    ncclComm_t comm = nullptr;
    int rank = 0;
    int world = 1;
    int timeout_ms = 60000;
    bool aborted = false;
};

struct geo_b200_trainer {
    int device = 0;
    geo::SignPlan plan;
    geo::RepDevice rep;
    bool rep_ok = false;
    int algorithm = GEO_B200_ALGORITHM_AUTO;
    int blades = 0;
    geo_b200_optimizer_config_t config;
    double *state = nullptr;     // [0,64) w, [64,128) m, [128,192) v, [192] loss sum, [200,272) rank record
    double *gather = nullptr;    // world * kRecStride
    double *records = nullptr;   // kMaxCtas * kRecStride
    uint32_t *status = nullptr;  // sticky device status word
    unsigned long long *dev_steps = nullptr;
    uint64_t host_steps = 0;     // steps assumed committed (resynchronised at sync)
    cudaStream_t last_stream = nullptr;
    geo_b200_comm_t *comm = nullptr;
    // host-buffer path
    cudaStream_t host_stream = nullptr;
    double *host_x = nullptr;
    double *host_t = nullptr;
    size_t host_cap = 0;
};

namespace {

// NCCL is resolved lazily with dlopen when the first communicator is made, so
// loading libgeo_b200.so never pulls an NCCL into the process: a host program
// (or a framework loaded later) keeps whichever NCCL it links itself, and an
// NCCL already present in the process is reused.
struct NcclApi {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
};

NcclApi load_nccl() {
    NcclApi api;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return api;
    api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    api.CommInitRankConfig = (decltype(api.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
    api.CommGetAsyncError = (decltype(api.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
    api.CommAbort = (decltype(api.CommAbort))dlsym(h, "ncclCommAbort");
    api.CommFinalize = (decltype(api.CommFinalize))dlsym(h, "ncclCommFinalize");
    api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
    api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
    api.loaded = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort &&
                 api.CommFinalize && api.CommDestroy && api.AllGather;
    return api;
}

NcclApi &nccl() {
    static NcclApi api = load_nccl();  // thread-safe one-time initialisation
    return api;
}

constexpr size_t kStateW = 0, kStateM = 64, kStateV = 128, kStateLoss = 192, kStateRecord = 200;
constexpr size_t kStateDoubles = kStateRecord + geo::kRecStride;

geo_b200_status_t from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return GEO_B200_OK;
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? GEO_B200_ALLOCATION_FAILURE : GEO_B200_RUNTIME_FAILURE;
}

bool config_valid(const geo_b200_optimizer_config_t *c) {
    return c != nullptr && (c->optimizer == GEO_B200_OPTIMIZER_SGD || c->optimizer == GEO_B200_OPTIMIZER_ADAM) &&
           isfinite(c->learning_rate) && c->learning_rate > 0.0 && isfinite(c->beta1) && c->beta1 >= 0.0 &&
           c->beta1 < 1.0 && isfinite(c->beta2) && c->beta2 >= 0.0 && c->beta2 < 1.0 && isfinite(c->epsilon) &&
           c->epsilon > 0.0;
}

// Wait for `stream`, polling NCCL for asynchronous errors when a communicator
// is attached; gives up after the communicator's timeout.
geo_b200_status_t wait_stream(cudaStream_t stream, geo_b200_comm_t *comm) {
    if (comm == nullptr) return from_cuda(cudaStreamSynchronize(stream));
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(stream);
        if (q == cudaSuccess) return GEO_B200_OK;
        if (q != cudaErrorNotReady) return from_cuda(q);
        ncclResult_t async = ncclSuccess;
        if (nccl().CommGetAsyncError(comm->comm, &async) != ncclSuccess ||
            (async != ncclSuccess && async != ncclInProgress)) {
            geo_b200_comm_abort(comm);
            return GEO_B200_COMM_FAILURE;
        }
        const auto waited =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - start).count();
        if (waited > comm->timeout_ms) {
            geo_b200_comm_abort(comm);
            return GEO_B200_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Non-blocking communicators may return ncclInProgress from a call; poll until
// it settles (bounded by the communicator timeout).
geo_b200_status_t nccl_settle(geo_b200_comm_t *comm, ncclResult_t r) {
    if (r == ncclSuccess) return GEO_B200_OK;
    if (r != ncclInProgress) return GEO_B200_COMM_FAILURE;
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t async = ncclInProgress;
        if (nccl().CommGetAsyncError(comm->comm, &async) != ncclSuccess) return GEO_B200_COMM_FAILURE;
        if (async == ncclSuccess) return GEO_B200_OK;
        if (async != ncclInProgress) return GEO_B200_COMM_FAILURE;
        const auto waited =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - start).count();
        if (waited > comm->timeout_ms) return GEO_B200_TIMEOUT;
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

geo_b200_status_t status_from_bits(uint32_t bits) {
    if (bits == 0u) return GEO_B200_OK;
    return GEO_B200_NUMERIC_FAILURE;
}

}  // namespace

extern "C" uint32_t geo_b200_abi_version(void) { return GEO_B200_ABI_VERSION; }

extern "C" const char *geo_b200_status_string(geo_b200_status_t status) {
    switch (status) {
        case GEO_B200_OK: return "ok";
        case GEO_B200_INVALID_ARGUMENT: return "invalid_argument";
        case GEO_B200_UNSUPPORTED_DIMENSION: return "unsupported_dimension";
        case GEO_B200_NUMERIC_FAILURE: return "numeric_failure";
        case GEO_B200_RUNTIME_FAILURE: return "runtime_failure";
        case GEO_B200_ALLOCATION_FAILURE: return "allocation_failure";
        case GEO_B200_COMM_FAILURE: return "comm_failure";
        case GEO_B200_TIMEOUT: return "timeout";
        default: return "unknown";
    }
}

extern "C" geo_b200_status_t geo_b200_trainer_create(geo_b200_trainer_t **out, uint8_t dimension,
                                                     const int8_t *signature, int parameter_on_left,
                                                     const double *initial_parameter,
                                                     const geo_b200_optimizer_config_t *config) {
    if (out == nullptr || signature == nullptr || initial_parameter == nullptr) return GEO_B200_INVALID_ARGUMENT;
    *out = nullptr;
    if (!geo::dimension_valid(dimension)) return GEO_B200_UNSUPPORTED_DIMENSION;
    if (!geo::signature_valid(signature, dimension) || !config_valid(config)) return GEO_B200_INVALID_ARGUMENT;
    const int blades = 1 << dimension;
    for (int b = 0; b < blades; ++b)
        if (!isfinite(initial_parameter[b])) return GEO_B200_INVALID_ARGUMENT;
    geo_b200_trainer_t *t = new (std::nothrow) geo_b200_trainer_t();
    if (t == nullptr) return GEO_B200_ALLOCATION_FAILURE;
    if (!geo::make_sign_plan(&t->plan, dimension, signature, parameter_on_left)) {
        delete t;
        return GEO_B200_INVALID_ARGUMENT;
    }
    t->blades = blades;
    t->config = *config;
    {
        geo::RepPlan rp;
        t->rep_ok = geo::make_rep_plan(&rp, dimension, signature, parameter_on_left) &&
                    geo::make_rep_device(&t->rep, rp) && geo::rep_supported(t->rep);
    }
    cudaGetDevice(&t->device);
    geo_b200_status_t st = GEO_B200_OK;
    double init[kStateDoubles];
    memset(init, 0, sizeof(init));
    memcpy(init + kStateW, initial_parameter, (size_t)blades * sizeof(double));
    if ((st = from_cuda(cudaMalloc((void **)&t->state, kStateDoubles * sizeof(double)))) != GEO_B200_OK ||
        (st = from_cuda(cudaMalloc((void **)&t->records,
                                   (size_t)geo::kMaxCtas * geo::kRecStride * sizeof(double)))) != GEO_B200_OK ||
        (st = from_cuda(cudaMalloc((void **)&t->status, 64))) != GEO_B200_OK ||
        (st = from_cuda(cudaMalloc((void **)&t->dev_steps, sizeof(unsigned long long)))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemcpy(t->state, init, sizeof(init), cudaMemcpyHostToDevice))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemset(t->status, 0, 64))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemset(t->dev_steps, 0, sizeof(unsigned long long)))) != GEO_B200_OK ||
        (st = from_cuda(cudaStreamCreateWithFlags(&t->host_stream, cudaStreamNonBlocking))) != GEO_B200_OK) {
        geo_b200_trainer_destroy(t);
        return st;
    }
    *out = t;
    return GEO_B200_OK;
}

extern "C" void geo_b200_trainer_destroy(geo_b200_trainer_t *t) {
    if (t == nullptr) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(t->device);
    if (t->host_stream) cudaStreamSynchronize(t->host_stream);
    if (t->last_stream) cudaStreamSynchronize(t->last_stream);
    cudaFree(t->state);
    cudaFree(t->gather);
    cudaFree(t->records);
    cudaFree(t->status);
    cudaFree(t->dev_steps);
    cudaFree(t->host_x);
    cudaFree(t->host_t);
    if (t->host_stream) cudaStreamDestroy(t->host_stream);
    cudaSetDevice(prev);
    delete t;
}

extern "C" geo_b200_status_t geo_b200_trainer_accumulate_device(geo_b200_trainer_t *t, const double *device_inputs,
                                                                const double *device_targets, size_t batch,
                                                                cudaStream_t stream) {
    geo::NvtxRange range("geo_b200.trainer.accumulate");
    if (t == nullptr || device_inputs == nullptr || device_targets == nullptr || batch == 0)
        return GEO_B200_INVALID_ARGUMENT;
    int ctas = 0;
    cudaError_t e;
    if (geo_b200_trainer_algorithm(t) == GEO_B200_ALGORITHM_REPRESENTATION)
        e = geo::launch_rep_cycle(t->rep, device_inputs, device_targets, t->state + kStateW, batch, t->records, &ctas,
                                  stream);
    else
        e = geo::launch_cycle(t->plan, geo::kCycle, device_inputs, device_targets, t->state + kStateW, nullptr,
                              batch, t->records, &ctas, stream);
    if (e == cudaSuccess) e = geo::launch_reduce_records(t->records, ctas, t->state + kStateRecord, stream, 1);
    t->last_stream = stream;
    return from_cuda(e);
}

extern "C" geo_b200_status_t geo_b200_trainer_apply(geo_b200_trainer_t *t, double gradient_scale,
                                                    cudaStream_t stream) {
    geo::NvtxRange range("geo_b200.trainer.apply");
    if (t == nullptr || !isfinite(gradient_scale) || gradient_scale <= 0.0) return GEO_B200_INVALID_ARGUMENT;
    geo::OptimizerArgs opt{};
    opt.kind = t->config.optimizer == GEO_B200_OPTIMIZER_ADAM ? geo::kOptAdamV8 : geo::kOptSgdV8;
    opt.blades = t->blades;
    opt.learning_rate = t->config.learning_rate;
    opt.beta1 = t->config.beta1;
    opt.beta2 = t->config.beta2;
    opt.epsilon = t->config.epsilon;
    opt.gradient_scale = gradient_scale;
    opt.batch_divisor = 1.0;
    opt.bias1 = 1.0;
    opt.bias2 = 1.0;
    if (opt.kind == geo::kOptAdamV8) {
        // reference src/full_cycle_v8.c:976-984, same libm pow
        const double step = (double)(t->host_steps + 1u);
        opt.bias1 = 1.0 - pow(t->config.beta1, step);
        opt.bias2 = 1.0 - pow(t->config.beta2, step);
        if (!isfinite(opt.bias1) || !isfinite(opt.bias2) || opt.bias1 <= 0.0 || opt.bias2 <= 0.0)
            return GEO_B200_NUMERIC_FAILURE;
    }
    const double *final_records = t->state + kStateRecord;
    int final_count = 1;
    if (t->comm != nullptr && t->comm->world > 1) {
        if (t->comm->aborted) return GEO_B200_COMM_FAILURE;
        const geo_b200_status_t s = nccl_settle(
            t->comm, nccl().AllGather(t->state + kStateRecord, t->gather, (size_t)geo::kRecStride, ncclDouble,
                                   t->comm->comm, stream));
        if (s != GEO_B200_OK) return s;
        final_records = t->gather;
        final_count = t->comm->world;
    }
    cudaError_t e = geo::launch_finalize(final_records, final_count, opt, nullptr, t->state + kStateLoss,
                                         t->state + kStateW, t->state + kStateM, t->state + kStateV, t->status,
                                         stream, t->dev_steps);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(t->state + kStateRecord, 0, geo::kRecStride * sizeof(double), stream);
    if (e != cudaSuccess) return from_cuda(e);
    t->host_steps += 1u;
    t->last_stream = stream;
    return GEO_B200_OK;
}

extern "C" geo_b200_status_t geo_b200_trainer_step_device(geo_b200_trainer_t *t, const double *device_inputs,
                                                          const double *device_targets, size_t batch,
                                                          double gradient_scale, cudaStream_t stream) {
    if (t == nullptr || !isfinite(gradient_scale) || gradient_scale <= 0.0) return GEO_B200_INVALID_ARGUMENT;
    const geo_b200_status_t st = geo_b200_trainer_accumulate_device(t, device_inputs, device_targets, batch, stream);
    if (st != GEO_B200_OK) return st;
    return geo_b200_trainer_apply(t, gradient_scale, stream);
}

extern "C" geo_b200_status_t geo_b200_trainer_sync(geo_b200_trainer_t *t, double *loss_sum) {
    geo::NvtxRange range("geo_b200.trainer.sync");
    if (t == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (t->last_stream != nullptr || t->comm != nullptr) {
        const geo_b200_status_t w = wait_stream(t->last_stream, t->comm);
        if (w != GEO_B200_OK) return w;
    }
    uint32_t bits = 0;
    unsigned long long steps = 0;
    double loss = 0.0;
    geo_b200_status_t st;
    if ((st = from_cuda(cudaMemcpy(&bits, t->status, sizeof(bits), cudaMemcpyDeviceToHost))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemcpy(&steps, t->dev_steps, sizeof(steps), cudaMemcpyDeviceToHost))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemcpy(&loss, t->state + kStateLoss, sizeof(loss), cudaMemcpyDeviceToHost))) !=
            GEO_B200_OK)
        return st;
    t->host_steps = steps;
    if (bits != 0u) cudaMemset(t->status, 0, sizeof(uint32_t));
    if (loss_sum) *loss_sum = loss;
    return status_from_bits(bits);
}

extern "C" geo_b200_status_t geo_b200_trainer_step_host(geo_b200_trainer_t *t, const double *inputs,
                                                        const double *targets, size_t batch, double gradient_scale,
                                                        double *loss_sum) {
    geo::NvtxRange range("geo_b200.trainer.step_host");
    if (t == nullptr || inputs == nullptr || targets == nullptr || batch == 0) return GEO_B200_INVALID_ARGUMENT;
    const size_t values = batch * (size_t)t->blades;
    const bool x_dev = geo::classify_pointer(inputs) == geo::Residency::kDevice;
    const bool t_dev = geo::classify_pointer(targets) == geo::Residency::kDevice;
    if ((!x_dev || !t_dev) && t->host_cap < values) {
        cudaFree(t->host_x);
        cudaFree(t->host_t);
        t->host_x = t->host_t = nullptr;
        t->host_cap = 0;
        geo_b200_status_t st;
        if ((st = from_cuda(cudaMalloc((void **)&t->host_x, values * sizeof(double)))) != GEO_B200_OK) return st;
        if ((st = from_cuda(cudaMalloc((void **)&t->host_t, values * sizeof(double)))) != GEO_B200_OK) return st;
        t->host_cap = values;
    }
    const double *dx = inputs, *dt = targets;
    if (!x_dev) {
        if (cudaMemcpyAsync(t->host_x, inputs, values * sizeof(double), cudaMemcpyDefault, t->host_stream) !=
            cudaSuccess)
            return from_cuda(cudaGetLastError());
        dx = t->host_x;
    }
    if (!t_dev) {
        if (cudaMemcpyAsync(t->host_t, targets, values * sizeof(double), cudaMemcpyDefault, t->host_stream) !=
            cudaSuccess)
            return from_cuda(cudaGetLastError());
        dt = t->host_t;
    }
    geo_b200_status_t st = geo_b200_trainer_step_device(t, dx, dt, batch, gradient_scale, t->host_stream);
    if (st != GEO_B200_OK) return st;
    return geo_b200_trainer_sync(t, loss_sum);
}

extern "C" geo_b200_status_t geo_b200_trainer_get_state(geo_b200_trainer_t *t, double *parameter,
                                                        double *first_moment, double *second_moment,
                                                        uint64_t *step_count) {
    if (t == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (t->last_stream) cudaStreamSynchronize(t->last_stream);
    double state[kStateDoubles];
    unsigned long long steps = 0;
    geo_b200_status_t st;
    if ((st = from_cuda(cudaMemcpy(state, t->state, sizeof(state), cudaMemcpyDeviceToHost))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemcpy(&steps, t->dev_steps, sizeof(steps), cudaMemcpyDeviceToHost))) != GEO_B200_OK)
        return st;
    const size_t bytes = (size_t)t->blades * sizeof(double);
    if (parameter) memcpy(parameter, state + kStateW, bytes);
    if (first_moment) memcpy(first_moment, state + kStateM, bytes);
    if (second_moment) memcpy(second_moment, state + kStateV, bytes);
    if (step_count) *step_count = steps;
    return GEO_B200_OK;
}

extern "C" geo_b200_status_t geo_b200_trainer_set_state(geo_b200_trainer_t *t, const double *parameter,
                                                        const double *first_moment, const double *second_moment,
                                                        uint64_t step_count) {
    if (t == nullptr || parameter == nullptr) return GEO_B200_INVALID_ARGUMENT;
    for (int b = 0; b < t->blades; ++b)
        if (!isfinite(parameter[b])) return GEO_B200_INVALID_ARGUMENT;
    if (t->last_stream) cudaStreamSynchronize(t->last_stream);
    double state[kStateDoubles];
    memset(state, 0, sizeof(state));
    const size_t bytes = (size_t)t->blades * sizeof(double);
    memcpy(state + kStateW, parameter, bytes);
    if (first_moment) memcpy(state + kStateM, first_moment, bytes);
    if (second_moment) memcpy(state + kStateV, second_moment, bytes);
    unsigned long long steps = step_count;
    geo_b200_status_t st;
    if ((st = from_cuda(cudaMemcpy(t->state, state, sizeof(state), cudaMemcpyHostToDevice))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemcpy(t->dev_steps, &steps, sizeof(steps), cudaMemcpyHostToDevice))) != GEO_B200_OK ||
        (st = from_cuda(cudaMemset(t->status, 0, sizeof(uint32_t)))) != GEO_B200_OK)
        return st;
    t->host_steps = step_count;
    return GEO_B200_OK;
}

extern "C" geo_b200_status_t geo_b200_trainer_set_parameter(geo_b200_trainer_t *t, const double *parameter) {
    return geo_b200_trainer_set_state(t, parameter, nullptr, nullptr, 0u);
}

extern "C" geo_b200_status_t geo_b200_trainer_set_algorithm(geo_b200_trainer_t *t, geo_b200_algorithm_t algorithm) {
    if (t == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (algorithm != GEO_B200_ALGORITHM_AUTO && algorithm != GEO_B200_ALGORITHM_CAYLEY &&
        algorithm != GEO_B200_ALGORITHM_REPRESENTATION)
        return GEO_B200_INVALID_ARGUMENT;
    if (algorithm == GEO_B200_ALGORITHM_REPRESENTATION && !t->rep_ok) return GEO_B200_INVALID_ARGUMENT;
    t->algorithm = algorithm;
    return GEO_B200_OK;
}

extern "C" geo_b200_algorithm_t geo_b200_trainer_algorithm(const geo_b200_trainer_t *t) {
    if (t == nullptr) return GEO_B200_ALGORITHM_AUTO;
    if (t->algorithm == GEO_B200_ALGORITHM_CAYLEY) return GEO_B200_ALGORITHM_CAYLEY;
    if (t->algorithm == GEO_B200_ALGORITHM_REPRESENTATION) return GEO_B200_ALGORITHM_REPRESENTATION;
    return (t->rep_ok && t->plan.dimension >= 5) ? GEO_B200_ALGORITHM_REPRESENTATION : GEO_B200_ALGORITHM_CAYLEY;
}

extern "C" const double *geo_b200_trainer_device_parameter(const geo_b200_trainer_t *t) {
    return t == nullptr ? nullptr : t->state + kStateW;
}

// ---- communicator ---------------------------------------------------------

static_assert(sizeof(ncclUniqueId) == GEO_B200_COMM_ID_BYTES, "NCCL unique id size");

extern "C" geo_b200_status_t geo_b200_comm_unique_id(unsigned char id[GEO_B200_COMM_ID_BYTES]) {
    if (id == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (!nccl().loaded) return GEO_B200_COMM_FAILURE;
    ncclUniqueId uid;
    if (nccl().GetUniqueId(&uid) != ncclSuccess) return GEO_B200_COMM_FAILURE;
    memcpy(id, &uid, sizeof(uid));
    return GEO_B200_OK;
}

extern "C" geo_b200_status_t geo_b200_comm_create(geo_b200_comm_t **out, int rank, int world,
                                                  const unsigned char id[GEO_B200_COMM_ID_BYTES], int timeout_ms) {
    if (out == nullptr || id == nullptr || world < 1 || rank < 0 || rank >= world || timeout_ms <= 0)
        return GEO_B200_INVALID_ARGUMENT;
    *out = nullptr;
    if (!nccl().loaded) return GEO_B200_COMM_FAILURE;
    geo_b200_comm_t *c = new (std::nothrow) geo_b200_comm_t();
    if (c == nullptr) return GEO_B200_ALLOCATION_FAILURE;
    c->rank = rank;
    c->world = world;
    c->timeout_ms = timeout_ms;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclResult_t r = nccl().CommInitRankConfig(&c->comm, world, uid, rank, &config);
    geo_b200_status_t st = GEO_B200_OK;
    if (r == ncclInProgress || r == ncclSuccess) {
        st = nccl_settle(c, r == ncclSuccess ? ncclInProgress : r);
    } else {
        st = GEO_B200_COMM_FAILURE;
    }
    if (st != GEO_B200_OK) {
        if (c->comm != nullptr) nccl().CommAbort(c->comm);
        delete c;
        return st;
    }
    *out = c;
    return GEO_B200_OK;
}

extern "C" void geo_b200_comm_abort(geo_b200_comm_t *c) {
    if (c == nullptr || c->comm == nullptr || c->aborted) return;
    nccl().CommAbort(c->comm);
    c->aborted = true;
}

extern "C" void geo_b200_comm_destroy(geo_b200_comm_t *c) {
    if (c == nullptr) return;
    if (c->comm != nullptr && !c->aborted) {
        ncclResult_t r = nccl().CommFinalize(c->comm);
        if (r == ncclInProgress) (void)nccl_settle(c, r);
        nccl().CommDestroy(c->comm);
    }
    delete c;
}

extern "C" geo_b200_status_t geo_b200_trainer_attach_comm(geo_b200_trainer_t *t, geo_b200_comm_t *c) {
    if (t == nullptr) return GEO_B200_INVALID_ARGUMENT;
    cudaFree(t->gather);
    t->gather = nullptr;
    t->comm = c;
    if (c != nullptr && c->world > 1) {
        const geo_b200_status_t st = from_cuda(
            cudaMalloc((void **)&t->gather, (size_t)c->world * geo::kRecStride * sizeof(double)));
        if (st != GEO_B200_OK) {
            t->comm = nullptr;
            return st;
        }
    }
    return GEO_B200_OK;
}
