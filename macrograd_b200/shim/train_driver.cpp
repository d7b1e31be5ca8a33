// train_driver.cpp -- the decoder-only character-model training step
// (6 layers, 6 heads, d_model 384, MLP 1536, context 256, vocab 65) built from
// the REFERENCE's own modules (mini_shakespeare/include/transformer.h:
// Transformer, Embedding, PositionalEmbedding, unmodified), its autograd, its
// cross-entropy loss and its AdamW, running on "cuda" with every matmul of
// the forward and backward pass served through the seam
// (kernel_ops_matmul.inc) by the sm_100a library -- or on "cpu", where the
// same step is the reference's own CPU arithmetic.
//
// C entry points for a host driver (macrograd_b200/training.py): build the
// model, draw a seeded batch, run forward + backward, move the parameter
// gradients through a flat buffer (for the data-parallel all-reduce), take
// the optimizer step. A seam observer times the step's GEMMs on the library
// stream and can capture chosen GEMMs' operands for the oracle.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "macrograd_nn.h"
#include "transformer.h"

extern "C" {
typedef struct mg_seam_call {
    void* out;
    const void* A;
    const void* B;
    const void* bias;
    int32_t rank;
    int32_t out_shape[16], A_shape[16], B_shape[16], bias_shape[16];
    int32_t transA, transB;
    void* stream;
} mg_seam_call;
typedef void (*mg_seam_observer)(int32_t phase, const mg_seam_call* call, void* ctx);
void mg_seam_set_observer(mg_seam_observer fn, void* ctx);
}

namespace {

// The module layout of the reference's MiniShakespeare
// (mini_shakespeare/include/mini_shakespeare.h:50-78): members constructed in
// this order (so the seeded initialisation draws in the same order), modules
// registered transformer, embedding, positional; the logits follow its
// internal_forward (mini_shakespeare.h:84-104). The dimensions are parameters.
class DecoderLM : public Module
{
public:
    Transformer transformer;
    PositionalEmbedding pos;
    Embedding embedding;

    DecoderLM(unsigned layers, unsigned heads, unsigned emb, unsigned ff, unsigned context, unsigned vocab)
        : transformer{layers, heads, emb, ff, 0.0f}, pos{context, emb}, embedding{vocab, emb}
    {
        add_module(transformer);
        add_module(embedding);
        add_module(pos);
    }

    Tensor logits(const VectorInt* tokens, unsigned batch)
    {
        Tensor token_emb = embedding.embed(tokens, batch);
        Tensor trans_in = pos(token_emb);
        Tensor mask = Functional::causal_mask(trans_in.size(1), device());
        transformer.set_attention_mask(mask);
        Tensor trans_out = transformer(trans_in);
        return embedding.unembed(trans_out);
    }
};

struct Captured {
    int32_t index = 0;
    mg_seam_call call{};
    std::vector<float> out, A, B, bias;
};

struct State {
    DecoderLM* model = nullptr;
    Optimizer::AdamW* opt = nullptr;
    std::vector<VectorInt> tokens;
    VectorInt targets;
    unsigned batch = 0, vocab = 0;
    bool gpu = false;
    // observer
    int mode = 0;                 // 0 off, 1 count and time, 2 capture
    int calls = 0;
    double flop = 0.0;
    std::vector<cudaEvent_t> ev;  // start / end per call
    std::vector<int32_t> want;    // call indices to capture
    std::vector<Captured> cap;
};

State* g = nullptr;

size_t numel(const int32_t* s, int32_t rank)
{
    size_t n = 1;
    for (int32_t i = 0; i < rank; ++i) n *= size_t(s[i]);
    return n;
}

double gemm_flop(const mg_seam_call& c)
{
    const int r = c.rank;
    double batch = 1.0;
    for (int i = 0; i < r - 2; ++i) batch *= c.out_shape[i];
    const double M = c.out_shape[r - 2], N = c.out_shape[r - 1];
    const double K = c.transA ? c.A_shape[r - 2] : c.A_shape[r - 1];
    return 2.0 * batch * M * N * K;
}

std::vector<float> to_host(const void* p, size_t n)
{
    std::vector<float> v(n);
    cudaMemcpy(v.data(), p, n * sizeof(float), cudaMemcpyDeviceToHost);
    return v;
}

void observe(int32_t phase, const mg_seam_call* c, void* /*ctx*/)
{
    State& s = *g;
    cudaStream_t st = static_cast<cudaStream_t>(c->stream);
    if (phase == 0) {
        if (s.mode == 1) {
            const size_t k = size_t(s.calls) * 2;
            while (s.ev.size() < k + 2) {
                cudaEvent_t e;
                cudaEventCreate(&e);
                s.ev.push_back(e);
            }
            cudaEventRecord(s.ev[k], st);
        }
        return;
    }
    if (s.mode == 1) cudaEventRecord(s.ev[size_t(s.calls) * 2 + 1], st);
    s.flop += gemm_flop(*c);
    if (s.mode == 2) {
        bool take = false;
        for (int32_t w : s.want) take = take || w == s.calls;
        if (take) {
            cudaStreamSynchronize(st);
            Captured k;
            k.index = s.calls;
            k.call = *c;
            k.out = to_host(c->out, numel(c->out_shape, c->rank));
            k.A = to_host(c->A, numel(c->A_shape, c->rank));
            k.B = to_host(c->B, numel(c->B_shape, c->rank));
            if (c->bias) k.bias = to_host(c->bias, numel(c->bias_shape, c->rank));
            s.cap.push_back(std::move(k));
        }
    }
    s.calls++;
}

// Parameter gradients of the model, in parameter-list order.
template <class F>
void for_each_param(F f)
{
    Tensor** p = g->model->get_parameters();
    const unsigned n = g->model->get_parameter_count();
    for (unsigned i = 0; i < n; ++i) f(*p[i]);
}

}  // namespace

extern "C" {

// Builds the model (seeded reference initialisation, on "cpu" then moved to
// `device`) and its AdamW optimizer. device_index >= 0 selects the GPU first.
int c5_create(int layers, int heads, int emb, int ff, int context, int vocab, unsigned long long seed,
              float lr, float weight_decay, const char* device, int device_index)
{
    if (g) return 1;
    if (device_index >= 0) Cuda::set_device(device_index);
    g = new State;
    g->gpu = std::strcmp(device, "cuda") == 0;
    g->vocab = unsigned(vocab);
    Random::set_seed(seed);
    g->model = new DecoderLM(unsigned(layers), unsigned(heads), unsigned(emb), unsigned(ff), unsigned(context),
                             unsigned(vocab));
    g->model->to(device);
    g->opt = new Optimizer::AdamW(*g->model, lr, weight_decay);
    return 0;
}

void c5_destroy(void)
{
    if (!g) return;
    mg_seam_set_observer(nullptr, nullptr);
    for (cudaEvent_t e : g->ev) cudaEventDestroy(e);
    delete g->opt;
    delete g->model;
    delete g;
    g = nullptr;
}

// Token ids and next-token targets for the whole batch (batch_total x T,
// uniform in [0, vocab) from the reference RNG: all token ids, then all
// targets), of which this process keeps sequences [first, first + count).
int c5_make_batch(unsigned long long seed, int batch_total, int T, int first, int count, int32_t* tokens_out,
                  int32_t* targets_out)
{
    if (!g || first < 0 || count < 1 || first + count > batch_total) return 1;
    Random::set_seed(seed);
    std::vector<int32_t> tok(size_t(batch_total) * T), tgt(size_t(batch_total) * T);
    for (auto& x : tok) x = Random::rand_int(0, int(g->vocab) - 1);
    for (auto& x : tgt) x = Random::rand_int(0, int(g->vocab) - 1);
    const char* dev = g->model->device();
    g->tokens.clear();
    for (int b = first; b < first + count; ++b) {
        VectorInt v(unsigned(T), "cpu");
        for (int t = 0; t < T; ++t) v[t] = tok[size_t(b) * T + t];
        g->tokens.push_back(v.to(dev));
    }
    VectorInt y(unsigned(count * T), "cpu");
    for (int i = 0; i < count * T; ++i) y[i] = tgt[size_t(first) * T + i];
    g->targets = y.to(dev);
    g->batch = unsigned(count);
    if (tokens_out) std::memcpy(tokens_out, tok.data() + size_t(first) * T, size_t(count) * T * 4);
    if (targets_out) std::memcpy(targets_out, tgt.data() + size_t(first) * T, size_t(count) * T * 4);
    return 0;
}

// zero_grad, forward, mean cross-entropy over this process's tokens, backward.
// Returns the loss.
float c5_forward_backward(void)
{
    g->model->with_grad();
    g->model->train();
    g->opt->zero_grad();
    Tensor logits = g->model->logits(g->tokens.data(), g->batch);
    Tensor loss = Functional::cross_entropy_loss(logits.view({-1, int(g->vocab)}), g->targets);
    loss.backward();
    return loss.item();
}

int c5_optimizer_step(void)
{
    g->opt->step();
    if (g->gpu) Cuda::synchronize();
    return 0;
}

void c5_synchronize(void)
{
    if (g && g->gpu) Cuda::synchronize();
}

int c5_param_count(void) { return g ? int(g->model->get_parameter_count()) : 0; }

long long c5_param_numel(void)
{
    long long n = 0;
    if (g) for_each_param([&](Tensor& t) { n += (long long)t.numel(); });
    return n;
}

// Element count of every parameter, in parameter-list order.
int c5_param_sizes(long long* out)
{
    if (!g) return 1;
    int i = 0;
    for_each_param([&](Tensor& t) { out[i++] = (long long)t.numel(); });
    return 0;
}

// All parameter gradients (which == 0) or parameter values (which == 1),
// flattened in parameter-list order, to dst (device memory of this GPU when
// the model is on "cuda", else host memory).
int c5_copy_out(int which, float* dst)
{
    if (!g) return 1;
    c5_synchronize();
    size_t off = 0;
    for_each_param([&](Tensor& t) {
        const float* src = which ? t.internal_data() : t.internal_gradient().internal_data();
        const size_t n = t.numel();
        if (g->gpu) cudaMemcpyAsync(dst + off, src, n * 4, cudaMemcpyDeviceToDevice, 0);
        else std::memcpy(dst + off, src, n * 4);
        off += n;
    });
    if (g->gpu) return cudaStreamSynchronize(0) == cudaSuccess ? 0 : 2;
    return 0;
}

// Overwrites the parameter gradients with src (same layout as c5_copy_out).
int c5_load_grads(const float* src)
{
    if (!g) return 1;
    c5_synchronize();
    size_t off = 0;
    for_each_param([&](Tensor& t) {
        float* d = t.internal_gradient().internal_data();
        const size_t n = t.numel();
        if (g->gpu) cudaMemcpyAsync(d, src + off, n * 4, cudaMemcpyDeviceToDevice, 0);
        else std::memcpy(d, src + off, n * 4);
        off += n;
    });
    if (g->gpu) return cudaStreamSynchronize(0) == cudaSuccess ? 0 : 2;
    return 0;
}

// Seam observer: mode 0 off, 1 count and time every GEMM (CUDA events on the
// library stream), 2 count and capture the operands of the calls listed.
int c5_observe(int mode, const int32_t* indices, int n)
{
    if (!g) return 1;
    g->mode = mode;
    g->calls = 0;
    g->flop = 0.0;
    g->want.assign(indices, indices + (indices ? n : 0));
    g->cap.clear();
    mg_seam_set_observer(mode ? observe : nullptr, nullptr);
    return 0;
}

int c5_calls(void) { return g ? g->calls : 0; }
double c5_gemm_flop(void) { return g ? g->flop : 0.0; }

// Sum of the device times of the GEMMs seen since c5_observe(1, ...).
double c5_gemm_ms(void)
{
    if (!g || g->mode != 1) return 0.0;
    c5_synchronize();
    double ms = 0.0;
    for (int i = 0; i < g->calls; ++i) {
        float t = 0.f;
        cudaEventElapsedTime(&t, g->ev[size_t(i) * 2], g->ev[size_t(i) * 2 + 1]);
        ms += t;
    }
    return ms;
}

int c5_captured(void) { return g ? int(g->cap.size()) : 0; }

// meta: [index, rank, transA, transB, has_bias, out[16], A[16], B[16], bias[16]]
int c5_capture_meta(int j, int32_t* meta)
{
    if (!g || j < 0 || j >= int(g->cap.size())) return 1;
    const Captured& k = g->cap[size_t(j)];
    meta[0] = k.index;
    meta[1] = k.call.rank;
    meta[2] = k.call.transA;
    meta[3] = k.call.transB;
    meta[4] = k.call.bias ? 1 : 0;
    std::memcpy(meta + 5, k.call.out_shape, 64);
    std::memcpy(meta + 21, k.call.A_shape, 64);
    std::memcpy(meta + 37, k.call.B_shape, 64);
    std::memcpy(meta + 53, k.call.bias_shape, 64);
    return 0;
}

int c5_capture_data(int j, float* out, float* A, float* B, float* bias)
{
    if (!g || j < 0 || j >= int(g->cap.size())) return 1;
    const Captured& k = g->cap[size_t(j)];
    std::memcpy(out, k.out.data(), k.out.size() * 4);
    std::memcpy(A, k.A.data(), k.A.size() * 4);
    std::memcpy(B, k.B.data(), k.B.size() * 4);
    if (bias && !k.bias.empty()) std::memcpy(bias, k.bias.data(), k.bias.size() * 4);
    return 0;
}

}  // extern "C"
