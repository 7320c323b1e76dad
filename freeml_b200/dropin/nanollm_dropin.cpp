// The FreeML NanoLLM model on B200 through the drop-in backend:
// Model<float, MatrixCUDA<float>> built exactly as Examples/NanoLLM/
// NanoLLM.cpp:268-358 (BuildOrLoadModel) builds Model<float, MatrixCPU<float>>,
// with only the matrix type changed.  FreeML's own code draws the weights
// (RandomUtils::GetGenerator(), ToolsLibrary/Tools.h:15-27) through the
// MatrixCUDA host mirror, so they are the reference's weights bit for bit;
// every operator of Model::Run then runs as an sm_100a kernel.
//
// Modes (raw little-endian binary files):
//   greedy  --prompt F --plen P --new N --out-tokens F --out-logits F [--graph 1]
//           the reference greedy loop (one full-window Model::Run per token,
//           argmax of row P+step-1 with the first-max rule of
//           NanoLLM.cpp:189-204); prints JSON with the host transfers and
//           kernel launches counted inside the Run calls and the time per
//           Run; --graph 1 records Model::Run once as a launch plan
//           (freeml_cuda::RunGraph) and replays it for every token
//   engine  --prompt F --plen P --new N --out-tokens F
//           the KV-cached decode engine (fml_lm_*) bound to this model's
//           weight matrices (device pointers taken from its Datablobs)
//   weights --out F    every parameter in the canonical order
//   train   --tokens F --iters N [--lr X] --out-losses F --out F
//           N NanoLLM training iterations (forward, loss, backward, AdamW)
// Shape flags: --vocab --ctx --d --heads --layers --wseed
#include <ModelLibrary/Model.h>
#include <LayerLibrary/Layers.h>
#include <LossLibrary/Losses.h>
#include <OptimiserLibrary/Optimisers.h>
#include <MatrixLibrary/MatrixBase_Functions.h>
#include <ToolsLibrary/Tools.h>

#include <freeml_b200/MatrixCUDA.h>
#include <freeml_b200/MatrixCUDA_Functions.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <vector>

using T = float;
using Mat = MatrixCUDA<float>;
using Mgr = MatrixManager<float, Mat>;
using Blob = Datablob<float, Mat>;

namespace {

struct Args
{
    std::map<std::string, std::string> kv;
    std::string get(const std::string& k) const
    {
        auto it = kv.find(k);
        return it == kv.end() ? std::string() : it->second;
    }
    uint32_t u(const std::string& k, uint32_t def) const
    {
        auto it = kv.find(k);
        return it == kv.end() ? def : (uint32_t)std::strtoul(it->second.c_str(), nullptr, 10);
    }
    bool has(const std::string& k) const { return kv.count(k) != 0; }
};

std::vector<uint32_t> ReadU32(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) { std::fprintf(stderr, "cannot open %s\n", path.c_str()); std::exit(2); }
    std::vector<char> b((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<uint32_t> v(b.size() / 4);
    std::memcpy(v.data(), b.data(), v.size() * 4);
    return v;
}

template <class V>
void WriteRaw(const std::string& path, const V& v)
{
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), v.size() * sizeof(v[0]));
}

struct Shape
{
    uint32_t V, C, d, H, L, wseed;
};

struct Built
{
    std::unique_ptr<Model<T, Mat>> model;
    Mgr::MatrixRef posInput, window;
};

// NanoLLM.cpp:268-358 and :383-399, inference flavour (initForTraining =
// false: the same weight draws, no gradient buffers), dropout 0, no bias.
Built Build(const Shape& s, bool train = false, float lr = 1e-4f)
{
    Mgr& inst = Mgr::Instance();
    RandomUtils::GetGenerator().seed(s.wseed);
    Built b;
    b.model = std::make_unique<Model<T, Mat>>();
    Model<T, Mat>* m = b.model.get();

    auto* tok = new Embedding<T, Mat>();
    tok->SetName("embedding_token");
    auto* tokBlob = InitEmbeddingBlob<T, Mat>(s.V, s.d, s.C, 1u, train);
    m->AddLayer(tok, tokBlob);
    auto* pos = new Embedding<T, Mat>();
    pos->SetName("embedding_pos");
    auto* posBlob = InitEmbeddingBlob<T, Mat>(s.C, s.d, s.C, 1u, train);
    m->AddLayer(pos, posBlob);
    auto* add = new AddLayer<T, Mat>();
    add->SetName("token_pos_add");
    m->AddLayer(add, InitAddBlob<T, Mat>(train));
    m->AddDependency(add, 0, tok, 0);
    m->AddDependency(add, 1, pos, 0);
    auto* drop = new DropoutLayer<T, Mat>();
    drop->SetName("embedding_dropout");
    m->AddLayer(drop, InitDropoutBlob<T, Mat>(0.0f, train));
    m->AddDependency(drop, 0, add, 0);
    std::vector<TransformerBlockLayer<T, Mat>*> blocks;
    for (uint32_t i = 0; i < s.L; ++i)
    {
        auto* blk = new TransformerBlockLayer<T, Mat>();
        blk->SetName("block_" + std::to_string(i));
        const float rs = 1.0f / std::sqrt(2.0f * static_cast<float>(s.L));
        m->AddLayer(blk, InitTransformerBlockBlob<T, Mat>(s.d, s.H, 0.0f, s.C, 1u, train, false, rs));
        m->AddDependency(blk, 0, i ? static_cast<Layer<T, Mat>*>(blocks[i - 1]) : drop, 0);
        blocks.push_back(blk);
    }
    auto* lnf = new LayerNorm<T, Mat>();
    lnf->SetName("ln_f");
    m->AddLayer(lnf, InitLayerNormBlob<T, Mat>(train, true, false));
    m->AddDependency(lnf, 0, blocks.back(), 0);
    auto* flat = new FlattenCopyLayer<T, Mat>();
    flat->SetName("ln_f_flatten");
    m->AddLayer(flat, InitFlattenCopyBlob<T, Mat>(train));
    m->AddDependency(flat, 0, lnf, 0);
    auto* head = new Dense<T, Identity<T>, Mat, true>();
    head->SetName("lm_head");
    auto* headBlob = InitDenseBlob<T, Mat>(s.V, s.d, s.C, train, true, false, true);
    Mat* headW = headBlob->GetMatrix<Mat>("Dense_Weights");
    headBlob->Set("Dense_Weights", inst.GetHandle(tokBlob->GetMatrix<Mat>("Embedding_Weights")));
    inst.RemoveMatrix(headW);
    m->AddLayer(head, headBlob);
    m->AddDependency(head, 0, flat, 0);
    m->SetFinalOutputLayer(head);
    if (train)  // NanoLLM.cpp:350-352
    {
        m->SetOptimiser(new AdamWOptimiser<T, Mat>(lr, 0.9f, 0.999f, 1e-8f, 0.01f));
        m->SetLoss(new CategoricalCrossEntropyWithLogits<T, Mat>());
    }
    m->SetExpectedInputDims({1u, s.C, 1u});
    m->Init();

    b.posInput = inst.AllocateMatrix({1u, s.C, 1u}, "Pos_Input");
    for (uint32_t t = 0; t < s.C; ++t) b.posInput->SetValue(0u, t, 0u, static_cast<T>(t));
    pos->SetInput(posBlob, b.posInput.get(), 0u);
    b.window = inst.AllocateMatrix({1u, s.C, 1u}, "Window");
    float* w = b.window->DataWrite();
    for (uint32_t t = 0; t < s.C; ++t) w[t] = 0.0f;
    return b;
}

struct LayerWeights
{
    Mat *tok, *pos, *lnf;
    std::vector<Mat*> ln0, wqkv, wproj, ln1, wfc, wmlp;
};

LayerWeights Weights(Model<T, Mat>* m, uint32_t L)
{
    LayerWeights w;
    w.tok = m->GetLayerBlob("embedding_token")->GetMatrix("Embedding_Weights");
    w.pos = m->GetLayerBlob("embedding_pos")->GetMatrix("Embedding_Weights");
    w.lnf = m->GetLayerBlob("ln_f")->GetMatrix("GammaScale");
    for (uint32_t i = 0; i < L; ++i)
    {
        Blob* blk = m->GetLayerBlob("block_" + std::to_string(i));
        Blob* att = blk->GetBlob("AttentionLayerData");
        w.ln0.push_back(blk->GetBlob("LayerNorm0Data")->GetMatrix("GammaScale"));
        w.wqkv.push_back(att->GetBlob("CSA_AttentionLayer")->GetMatrix("Dense_Weights"));
        w.wproj.push_back(att->GetBlob("CSA_ProjLayer")->GetMatrix("Dense_Weights"));
        w.ln1.push_back(blk->GetBlob("LayerNorm1Data")->GetMatrix("GammaScale"));
        w.wfc.push_back(blk->GetBlob("DenseFCData")->GetMatrix("Dense_Weights"));
        w.wmlp.push_back(blk->GetBlob("DenseProjData")->GetMatrix("Dense_Weights"));
    }
    return w;
}

int Greedy(const Shape& s, const Args& a)
{
    const uint32_t plen = a.u("plen", 16), nnew = a.u("new", 112);
    std::vector<uint32_t> prompt = ReadU32(a.get("prompt"));
    if (prompt.size() < plen || plen + nnew > s.C) { std::fprintf(stderr, "bad prompt/new\n"); return 2; }
    Built b = Build(s);
    std::vector<uint32_t> tokens(prompt.begin(), prompt.begin() + plen);
    std::vector<float> rows;
    float* win = b.window->DataWrite();
    for (uint32_t t = 0; t < plen; ++t) win[t] = (float)tokens[t];
    // one untimed Run uploads the host-written init data (weights drawn by
    // FreeML's own init code, masks, scalars, positions)
    b.window->Flush();
    b.model->Run(b.window.get(), nullptr);
    fml_synchronize();
    // --graph 1: Model::Run recorded once as a launch plan and replayed
    const bool graph = a.u("graph", 0) != 0;
    freeml_cuda::RunGraph plan;
    if (graph) plan.Record([&] { b.model->Run(b.window.get(), nullptr); });
    uint64_t run_transfers = 0, run_launches = 0;
    double run_seconds = 0.0;
    for (uint32_t step = 0; step < nnew; ++step)
    {
        b.window->Flush();
        fml_synchronize();
        const auto t0 = Mat::HostTransfers();
        const uint64_t l0 = fml_kernel_launch_count();
        const auto c0 = std::chrono::steady_clock::now();
        if (graph) plan.Replay();
        else b.model->Run(b.window.get(), nullptr);
        fml_synchronize();
        run_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - c0).count();
        const auto t1 = Mat::HostTransfers();
        run_launches += fml_kernel_launch_count() - l0;
        run_transfers += (t1.downloads - t0.downloads) + (t1.uploads - t0.uploads);
        Mat* logits = b.model->GetOutput();
        const uint32_t r = plen + step - 1u;
        const float* row = logits->DataRead() + (size_t)r * logits->GetDimsX();
        uint32_t best = 0;
        float bv = row[0];
        for (uint32_t v = 1; v < s.V; ++v)
            if (row[v] > bv) { bv = row[v]; best = v; }
        rows.insert(rows.end(), row, row + s.V);
        tokens.push_back(best);
        b.window->DataWrite()[r + 1] = (float)best;
    }
    WriteRaw(a.get("out-tokens"), tokens);
    if (a.has("out-logits")) WriteRaw(a.get("out-logits"), rows);
    std::printf("{\"runs\": %u, \"graph\": %d, \"host_transfers_in_run\": %llu, \"kernel_launches_in_run\": %llu, "
                "\"ms_per_run\": %.4f}\n",
                nnew, graph ? 1 : 0, (unsigned long long)run_transfers, (unsigned long long)run_launches,
                1e3 * run_seconds / nnew);
    return 0;
}

int Engine(const Shape& s, const Args& a)
{
    const uint32_t plen = a.u("plen", 16), nnew = a.u("new", 112);
    std::vector<uint32_t> prompt = ReadU32(a.get("prompt"));
    if (prompt.size() < plen || plen + nnew > s.C) { std::fprintf(stderr, "bad prompt/new\n"); return 2; }
    Built b = Build(s);
    LayerWeights lw = Weights(b.model.get(), s.L);
    auto dev = [](Mat* m) { return m->DevIn(); };
    std::vector<const float*> ln0, wqkv, wproj, ln1, wfc, wmlp;
    for (uint32_t i = 0; i < s.L; ++i)
    {
        ln0.push_back(dev(lw.ln0[i])); wqkv.push_back(dev(lw.wqkv[i])); wproj.push_back(dev(lw.wproj[i]));
        ln1.push_back(dev(lw.ln1[i])); wfc.push_back(dev(lw.wfc[i])); wmlp.push_back(dev(lw.wmlp[i]));
    }
    fml_lm_weights w{dev(lw.tok), dev(lw.pos), ln0.data(), wqkv.data(), wproj.data(), ln1.data(), wfc.data(),
                     wmlp.data(), dev(lw.lnf)};
    fml_lm_config cfg{s.V, s.C, s.d, s.H, s.L, 1};
    fml_lm* lm = nullptr;
    freeml_cuda::Check(fml_lm_create(&cfg, 0, &lm), "fml_lm_create");
    freeml_cuda::Check(fml_lm_bind_weights(lm, &w, nullptr), "fml_lm_bind_weights");
    uint32_t* dprompt = nullptr;
    freeml_cuda::Check(fml_device_alloc(reinterpret_cast<void**>(&dprompt), plen * 4), "fml_device_alloc");
    freeml_cuda::Check(fml_memcpy_to_device(dprompt, prompt.data(), plen * 4), "fml_memcpy_to_device");
    freeml_cuda::Check(fml_lm_prefill(lm, dprompt, 1, plen, nullptr), "fml_lm_prefill");
    std::vector<uint32_t> tokens(prompt.begin(), prompt.begin() + plen);
    uint32_t* dnext = nullptr;
    freeml_cuda::Check(fml_device_alloc(reinterpret_cast<void**>(&dnext), 4), "fml_device_alloc");
    freeml_cuda::Check(fml_lm_pending(lm, dnext, nullptr), "fml_lm_pending");
    uint32_t tok = 0;
    freeml_cuda::Check(fml_memcpy_to_host(&tok, dnext, 4), "fml_memcpy_to_host");
    tokens.push_back(tok);
    for (uint32_t step = 1; step < nnew; ++step)
    {
        uint32_t out = 0;
        freeml_cuda::Check(fml_lm_step_host(lm, &tok, &out, nullptr), "fml_lm_step_host");
        tokens.push_back(out);
        tok = out;
    }
    WriteRaw(a.get("out-tokens"), tokens);
    fml_lm_destroy(lm);
    fml_device_free(dprompt);
    fml_device_free(dnext);
    std::printf("{\"engine_tokens\": %zu}\n", tokens.size());
    return 0;
}

std::vector<float> PackWeights(Built& b, const Shape& s)
{
    LayerWeights lw = Weights(b.model.get(), s.L);
    std::vector<float> out;
    auto app = [&](Mat* m) { const float* p = m->DataRead(); out.insert(out.end(), p, p + m->GetElementCount()); };
    app(lw.tok);
    app(lw.pos);
    for (uint32_t i = 0; i < s.L; ++i)
    {
        app(lw.ln0[i]); app(lw.wqkv[i]); app(lw.wproj[i]); app(lw.ln1[i]); app(lw.wfc[i]); app(lw.wmlp[i]);
    }
    app(lw.lnf);
    return out;
}

int DumpWeights(const Shape& s, const Args& a)
{
    Built b = Build(s);
    WriteRaw(a.get("out"), PackWeights(b, s));
    return 0;
}

// NanoLLM's training iteration (NanoLLM.cpp:404-440): Model::Run(window,
// target) = forward, CategoricalCrossEntropyWithLogits gradient and loss,
// backward, AdamW step, on consecutive windows of the stream --tokens F
// (C + iters ids): iteration i trains on [i, i + C) -> [i + 1, i + C + 1).
// Writes the losses (float64) and the parameters after the last step;
// prints the host transfers and kernel launches inside the Run calls after
// the first (which also uploads the host-written init data) and their time
// per iteration.
int Train(const Shape& s, const Args& a)
{
    const uint32_t iters = a.u("iters", 2);
    const float lr = a.has("lr") ? std::strtof(a.get("lr").c_str(), nullptr) : 1e-4f;
    std::vector<uint32_t> toks = ReadU32(a.get("tokens"));
    if (toks.size() < (size_t)s.C + iters) { std::fprintf(stderr, "need C + iters tokens\n"); return 2; }
    Built b = Build(s, true, lr);
    auto target = Mgr::Instance().AllocateMatrix({1u, s.C, 1u}, "Target");
    std::vector<double> losses;
    uint64_t transfers = 0, launches = 0;
    double seconds = 0.0;
    for (uint32_t it = 0; it < iters; ++it)
    {
        float* w = b.window->DataWrite();
        float* tg = target->DataWrite();
        for (uint32_t t = 0; t < s.C; ++t)
        {
            w[t] = (float)toks[it + t];
            tg[t] = (float)toks[it + t + 1];
        }
        b.window->Flush();
        target->Flush();
        fml_synchronize();
        const auto t0 = Mat::HostTransfers();
        const uint64_t l0 = fml_kernel_launch_count();
        const auto c0 = std::chrono::steady_clock::now();
        b.model->Run(b.window.get(), target.get(), true);
        fml_synchronize();
        if (it > 0) seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - c0).count();
        const auto t1 = Mat::HostTransfers();
        if (it > 0)  // the first Run also uploads the host-written init data
        {
            launches += fml_kernel_launch_count() - l0;
            transfers += (t1.downloads - t0.downloads) + (t1.uploads - t0.uploads);
        }
        losses.push_back(b.model->GetLastLoss());
    }
    if (a.has("out-losses")) WriteRaw(a.get("out-losses"), losses);
    if (a.has("out")) WriteRaw(a.get("out"), PackWeights(b, s));
    std::printf("{\"iters\": %u, \"host_transfers_in_run\": %llu, \"kernel_launches_in_run\": %llu, "
                "\"ms_per_iter\": %.4f}\n",
                iters, (unsigned long long)transfers, (unsigned long long)launches,
                iters > 1 ? 1e3 * seconds / (iters - 1) : 0.0);
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    Tools::Logger::SetMinLevel(Tools::Logger::Level::Error);
    if (argc < 2) { std::fprintf(stderr, "usage: %s greedy|engine|weights|train [--key value]...\n", argv[0]); return 2; }
    Args a;
    for (int i = 2; i + 1 < argc; i += 2)
        if (std::string(argv[i]).rfind("--", 0) == 0) a.kv[std::string(argv[i]).substr(2)] = argv[i + 1];
    Shape s{a.u("vocab", 256), a.u("ctx", 128), a.u("d", 128), a.u("heads", 4), a.u("layers", 4), a.u("wseed", 0)};
    const std::string mode = argv[1];
    // --math fp32|tf32x3|tf32: precision of the batched contractions (Mul,
    // MatMul_Strided above 64 rows); the library's default is tf32x3
    if (a.has("math"))
    {
        const std::string m = a.get("math");
        const int mm = m == "fp32" ? FML_MATH_FP32 : m == "tf32" ? FML_MATH_TF32 : FML_MATH_TF32X3;
        if (fml_set_math_mode(mm) != FML_OK) { std::fprintf(stderr, "%s\n", fml_last_error()); return 2; }
    }
    if (mode == "greedy") return Greedy(s, a);
    if (mode == "engine") return Engine(s, a);
    if (mode == "weights") return DumpWeights(s, a);
    if (mode == "train") return Train(s, a);
    std::fprintf(stderr, "unknown mode %s\n", mode.c_str());
    return 2;
}
