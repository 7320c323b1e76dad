// Test infrastructure: drives the UNMODIFIED FreeML reference CPU path
// (Model<float, MatrixCPU<float>>) so that its outputs can pin the oracle and
// the CUDA backend.  Compiled by oracle/Makefile against the reference tree;
// the binary lands in oracle/_ref/.  Nothing in the product links or runs it.
//
// The model is assembled exactly as Examples/NanoLLM/NanoLLM.cpp:268-358
// (BuildOrLoadModel) does it, minus checkpoint loading, optimiser and loss
// (Model::Run with target == nullptr never touches them, Model.h:764-788):
//   embedding_token  InitEmbeddingBlob(V, d, C, 1)          NanoLLM.cpp:276-279
//   embedding_pos    InitEmbeddingBlob(C, d, C, 1)          NanoLLM.cpp:282-285
//   token_pos_add, embedding_dropout (p = 0)                NanoLLM.cpp:288-300
//   block_i          InitTransformerBlockBlob(..., 1/sqrt(2L)) NanoLLM.cpp:303-318
//   ln_f, ln_f_flatten, lm_head (tied to the token table)   NanoLLM.cpp:321-348
// Weights come from RandomUtils::GetGenerator() seeded with --wseed before the
// first blob is built (ToolsLibrary/Tools.h:15-19).  The position input is
// 0..C-1 (NanoLLM.cpp:383-399).
//
// Prompt recipe (shared with tests/ and bench.py, which use numpy's legacy
// RandomState(seed).randint(0, V, n) -- the same stream): std::mt19937(pseed),
// each token = first (u32 & mask) <= V-1, mask = 2^ceil(log2 V) - 1, drawn
// sequence-major for B sequences.
//
// Modes (all binary files are raw little-endian):
//   weights  --out F            every parameter, canonical order (see DumpWeights)
//   greedy   --prompt F|--pseed S --plen P --new N --out-tokens F --out-logits F
//            the reference greedy loop: one full-window Model::Run per token,
//            argmax (strict '>') of logits row (P+step-1), NanoLLM.cpp:189-204
//   forward  --window F --out-logits F    one Run over a C-token window, all C rows
//   time     --forwards K --warmup W      seconds per full-window Run (JSON line)
//   op       --op NAME --in F --out F ... one generic operator on given inputs
//   save     --dir D --name N             Model::Save of the built model into D/N
//   train    --iters N --pseed S [--lr X] --out-losses F --out F
//            N training iterations of Model::Run(window, target)
#include <ModelLibrary/Model.h>
#include <LayerLibrary/Layers.h>
#include <LossLibrary/Losses.h>
#include <OptimiserLibrary/Optimisers.h>
#include <MatrixLibrary/CPU/MatrixCPU.h>
#include <MatrixLibrary/MatrixBase_Functions.h>
#include <MatrixLibrary/MatrixBase_Mul.h>
#include <ToolsLibrary/Tools.h>
#include <ToolsLibrary/ThreadPool.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <memory>
#include <random>
#include <string>
#include <vector>

using T = float;
using Mat = MatrixCPU<float>;
using Mgr = MatrixManager<float, Mat>;
using Blob = Datablob<float, Mat>;

struct Args
{
    std::map<std::string, std::string> kv;
    std::string get(const std::string& k, const std::string& def = "") const
    {
        auto it = kv.find(k);
        return it == kv.end() ? def : it->second;
    }
    uint32_t u(const std::string& k, uint32_t def = 0) const
    {
        auto it = kv.find(k);
        return it == kv.end() ? def : (uint32_t)std::strtoul(it->second.c_str(), nullptr, 10);
    }
    bool has(const std::string& k) const { return kv.count(k) != 0; }
};

static Args ParseArgs(int argc, char** argv, int first)
{
    Args a;
    for (int i = first; i < argc; ++i)
    {
        std::string k = argv[i];
        if (k.rfind("--", 0) == 0 && i + 1 < argc)
        {
            a.kv[k.substr(2)] = argv[i + 1];
            ++i;
        }
    }
    return a;
}

static std::vector<float> ReadF32(const std::string& path, size_t expect = 0)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) { std::fprintf(stderr, "cannot open %s\n", path.c_str()); std::exit(2); }
    std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<float> v(bytes.size() / 4);
    std::memcpy(v.data(), bytes.data(), v.size() * 4);
    if (expect && v.size() != expect) { std::fprintf(stderr, "%s: %zu floats, expected %zu\n", path.c_str(), v.size(), expect); std::exit(2); }
    return v;
}

static std::vector<uint32_t> ReadU32(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) { std::fprintf(stderr, "cannot open %s\n", path.c_str()); std::exit(2); }
    std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<uint32_t> v(bytes.size() / 4);
    std::memcpy(v.data(), bytes.data(), v.size() * 4);
    return v;
}

template<class V>
static void WriteRaw(const std::string& path, const V& v)
{
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), v.size() * sizeof(v[0]));
}

struct LMConfig
{
    uint32_t V = 256, C = 128, d = 128, H = 4, L = 4;
    uint32_t wseed = 0;
};

static LMConfig ConfigFrom(const Args& a)
{
    LMConfig c;
    c.V = a.u("vocab", 256);
    c.C = a.u("ctx", 128);
    c.d = a.u("d", 128);
    c.H = a.u("heads", 4);
    c.L = a.u("layers", 4);
    c.wseed = a.u("wseed", 0);
    return c;
}

struct Built
{
    std::unique_ptr<Model<T, Mat>> model;
    Mgr::MatrixRef posInput;
    Mgr::MatrixRef window;
};

// Mirrors BuildOrLoadModel (NanoLLM.cpp:268-358) and AllocateTrainingMatrices
// (NanoLLM.cpp:383-399) for inference: initForTraining = false (the same
// weight draws, no gradient buffers), dropout 0, use_bias false.
static Built BuildModel(const LMConfig& cfg, bool train = false, float lr = 1e-4f)
{
    Mgr& inst = Mgr::Instance();
    RandomUtils::GetGenerator().seed(cfg.wseed);
    Built b;
    b.model = std::make_unique<Model<T, Mat>>();
    Model<T, Mat>* model = b.model.get();

    auto* embTok = new Embedding<T, Mat>();
    embTok->SetName("embedding_token");
    auto* embTokBlob = InitEmbeddingBlob<T, Mat>(cfg.V, cfg.d, cfg.C, 1u, train);
    model->AddLayer(embTok, embTokBlob);

    auto* embPos = new Embedding<T, Mat>();
    embPos->SetName("embedding_pos");
    auto* embPosBlob = InitEmbeddingBlob<T, Mat>(cfg.C, cfg.d, cfg.C, 1u, train);
    model->AddLayer(embPos, embPosBlob);

    auto* add = new AddLayer<T, Mat>();
    add->SetName("token_pos_add");
    model->AddLayer(add, InitAddBlob<T, Mat>(train));
    model->AddDependency(add, 0, embTok, 0);
    model->AddDependency(add, 1, embPos, 0);

    auto* drop = new DropoutLayer<T, Mat>();
    drop->SetName("embedding_dropout");
    model->AddLayer(drop, InitDropoutBlob<T, Mat>(0.0f, train));
    model->AddDependency(drop, 0, add, 0);

    std::vector<TransformerBlockLayer<T, Mat>*> blocks;
    for (uint32_t i = 0; i < cfg.L; ++i)
    {
        auto* block = new TransformerBlockLayer<T, Mat>();
        block->SetName("block_" + std::to_string(i));
        const float residProjScale = 1.0f / std::sqrt(2.0f * static_cast<float>(cfg.L));
        auto* blob = InitTransformerBlockBlob<T, Mat>(cfg.d, cfg.H, 0.0f, cfg.C, 1u, train, false, residProjScale);
        model->AddLayer(block, blob);
        if (i != 0) model->AddDependency(block, 0, blocks[i - 1], 0);
        else        model->AddDependency(block, 0, drop, 0);
        blocks.push_back(block);
    }

    auto* lnf = new LayerNorm<T, Mat>();
    lnf->SetName("ln_f");
    model->AddLayer(lnf, InitLayerNormBlob<T, Mat>(train, true, false));
    model->AddDependency(lnf, 0, blocks.back(), 0);

    auto* flat = new FlattenCopyLayer<T, Mat>();
    flat->SetName("ln_f_flatten");
    model->AddLayer(flat, InitFlattenCopyBlob<T, Mat>(train));
    model->AddDependency(flat, 0, lnf, 0);

    auto* head = new Dense<T, Identity<T>, Mat, true>();
    head->SetName("lm_head");
    auto* headBlob = InitDenseBlob<T, Mat>(cfg.V, cfg.d, cfg.C, train, true, false, true);
    Mat* headW = headBlob->GetMatrix<Mat>("Dense_Weights");
    Mat* tokW = embTokBlob->GetMatrix<Mat>("Embedding_Weights");
    headBlob->Set("Dense_Weights", inst.GetHandle(tokW));
    inst.RemoveMatrix(headW);
    model->AddLayer(head, headBlob);
    model->AddDependency(head, 0, flat, 0);
    model->SetFinalOutputLayer(head);

    if (train)  // NanoLLM.cpp:350-352
    {
        model->SetOptimiser(new AdamWOptimiser<T, Mat>(lr, 0.9f, 0.999f, 1e-8f, 0.01f));
        model->SetLoss(new CategoricalCrossEntropyWithLogits<T, Mat>());
    }
    model->SetExpectedInputDims({1u, cfg.C, 1u});
    model->Init();

    b.posInput = inst.AllocateMatrix({1u, cfg.C, 1u}, "Pos_Input");
    for (uint32_t t = 0; t < cfg.C; ++t) b.posInput->SetValue(0u, t, 0u, static_cast<T>(t));
    embPos->SetInput(embPosBlob, b.posInput.get(), 0u);

    b.window = inst.AllocateMatrix({1u, cfg.C, 1u}, "Window");
    Fill(b.window.get(), 0.0f);
    return b;
}

static void AppendMatrix(std::vector<float>& out, Mat* m)
{
    const float* p = m->DataRead();
    out.insert(out.end(), p, p + m->GetElementCount());
}

// Canonical parameter order, shared with the oracle and the CUDA engine:
// tok_emb[V*d], pos_emb[C*d], per layer {ln0_gamma[d], w_qkv[d*3d],
// w_attn_proj[d*d] (stored out x in), ln1_gamma[d], w_fc[d*4d], w_mlp_proj[4d*d]},
// lnf_gamma[d].
static std::vector<float> DumpWeights(Built& b, const LMConfig& cfg)
{
    std::vector<float> out;
    Model<T, Mat>* m = b.model.get();
    AppendMatrix(out, m->GetLayerBlob("embedding_token")->GetMatrix("Embedding_Weights"));
    AppendMatrix(out, m->GetLayerBlob("embedding_pos")->GetMatrix("Embedding_Weights"));
    for (uint32_t i = 0; i < cfg.L; ++i)
    {
        Blob* blk = m->GetLayerBlob("block_" + std::to_string(i));
        AppendMatrix(out, blk->GetBlob("LayerNorm0Data")->GetMatrix("GammaScale"));
        Blob* att = blk->GetBlob("AttentionLayerData");
        AppendMatrix(out, att->GetBlob("CSA_AttentionLayer")->GetMatrix("Dense_Weights"));
        AppendMatrix(out, att->GetBlob("CSA_ProjLayer")->GetMatrix("Dense_Weights"));
        AppendMatrix(out, blk->GetBlob("LayerNorm1Data")->GetMatrix("GammaScale"));
        AppendMatrix(out, blk->GetBlob("DenseFCData")->GetMatrix("Dense_Weights"));
        AppendMatrix(out, blk->GetBlob("DenseProjData")->GetMatrix("Dense_Weights"));
    }
    AppendMatrix(out, m->GetLayerBlob("ln_f")->GetMatrix("GammaScale"));
    return out;
}

static std::vector<uint32_t> PromptTokens(uint32_t seed, uint32_t V, size_t n)
{
    std::mt19937 g(seed);
    uint32_t mask = 1;
    while (mask < V - 1u) mask = (mask << 1) | 1u;
    if (V == 1u) mask = 0u;
    std::vector<uint32_t> out(n);
    for (size_t i = 0; i < n; ++i)
    {
        uint32_t v;
        do { v = (uint32_t)g() & mask; } while (v > V - 1u);
        out[i] = v;
    }
    return out;
}

static void RunWindow(Built& b)
{
    b.model->Run(b.window.get(), nullptr);
}

static int ModeGreedy(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    const uint32_t plen = a.u("plen", 16), nnew = a.u("new", 112);
    std::vector<uint32_t> prompt = a.has("prompt") ? ReadU32(a.get("prompt"))
                                                   : PromptTokens(a.u("pseed", 1), cfg.V, plen);
    if (prompt.size() < plen || plen + nnew > cfg.C) { std::fprintf(stderr, "bad prompt/new sizes\n"); return 2; }
    Built b = BuildModel(cfg);
    std::vector<uint32_t> tokens(prompt.begin(), prompt.begin() + plen);
    std::vector<float> rows;
    rows.reserve((size_t)nnew * cfg.V);
    float* win = b.window->DataWrite();
    for (uint32_t t = 0; t < cfg.C; ++t) win[t] = t < plen ? (float)tokens[t] : 0.0f;
    for (uint32_t step = 0; step < nnew; ++step)
    {
        RunWindow(b);
        Mat* logits = b.model->GetOutput();
        const uint32_t r = plen + step - 1u;
        const float* row = logits->DataRead() + (size_t)r * logits->GetDimsX();
        uint32_t best = 0; float bestv = row[0];
        for (uint32_t v = 1; v < cfg.V; ++v) if (row[v] > bestv) { bestv = row[v]; best = v; }
        rows.insert(rows.end(), row, row + cfg.V);
        tokens.push_back(best);
        win[r + 1] = (float)best;
    }
    if (a.has("out-tokens")) WriteRaw(a.get("out-tokens"), tokens);
    if (a.has("out-logits")) WriteRaw(a.get("out-logits"), rows);
    return 0;
}

static int ModeForward(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    std::vector<uint32_t> w = ReadU32(a.get("window"));
    if (w.size() != cfg.C) { std::fprintf(stderr, "window must hold C tokens\n"); return 2; }
    Built b = BuildModel(cfg);
    float* win = b.window->DataWrite();
    for (uint32_t t = 0; t < cfg.C; ++t) win[t] = (float)w[t];
    RunWindow(b);
    Mat* logits = b.model->GetOutput();
    std::vector<float> out(logits->DataRead(), logits->DataRead() + logits->GetElementCount());
    WriteRaw(a.get("out-logits"), out);
    return 0;
}

static int ModeWeights(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    Built b = BuildModel(cfg);
    WriteRaw(a.get("out"), DumpWeights(b, cfg));
    return 0;
}

// NanoLLM's training iteration (NanoLLM.cpp:404-440: Model::Run(input,
// target) = forward, CategoricalCrossEntropyWithLogits gradient and loss,
// backward, AdamW step) on consecutive windows of one seeded token stream:
// iteration i trains on tokens [i, i + C) -> [i + 1, i + C + 1).  Writes the
// per-iteration losses (float64) and the parameters after the last step.
static int ModeTrain(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    const uint32_t iters = a.u("iters", 2);
    const float lr = a.has("lr") ? std::strtof(a.get("lr").c_str(), nullptr) : 1e-4f;
    Built b = BuildModel(cfg, true, lr);
    const std::vector<uint32_t> toks = PromptTokens(a.u("pseed", 1), cfg.V, (size_t)cfg.C + iters);
    auto target = Mgr::Instance().AllocateMatrix({1u, cfg.C, 1u}, "Target");
    std::vector<double> losses;
    for (uint32_t it = 0; it < iters; ++it)
    {
        float* w = b.window->DataWrite();
        float* tg = target->DataWrite();
        for (uint32_t t = 0; t < cfg.C; ++t)
        {
            w[t] = (float)toks[it + t];
            tg[t] = (float)toks[it + t + 1];
        }
        b.model->Run(b.window.get(), target.get(), true);
        losses.push_back(b.model->GetLastLoss());
    }
    if (a.has("out-losses")) WriteRaw(a.get("out-losses"), losses);
    if (a.has("out")) WriteRaw(a.get("out"), DumpWeights(b, cfg));
    return 0;
}

// The model saved by FreeML's own Model::Save (Model.h:91-159, SaveLoader.h:
// 499-577, 1523-1563) into <dir>/<name>: model.guide, one .blob_layer text file
// per (sub)layer, .blob_matrix headers and raw .blob_data payloads.
static int ModeSave(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    Built b = BuildModel(cfg);
    b.model->SetName(a.get("name", "nanollm"));
    const std::filesystem::path old = std::filesystem::current_path();
    std::filesystem::create_directories(a.get("dir", "."));
    std::filesystem::current_path(a.get("dir", "."));
    const bool ok = b.model->Save();
    std::filesystem::current_path(old);
    return ok ? 0 : 1;
}

static int ModeTime(const Args& a)
{
    LMConfig cfg = ConfigFrom(a);
    const uint32_t K = a.u("forwards", 3), W = a.u("warmup", 1);
    auto t0 = std::chrono::steady_clock::now();
    Built b = BuildModel(cfg);
    double build_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::vector<uint32_t> prompt = PromptTokens(a.u("pseed", 1), cfg.V, cfg.C);
    float* win = b.window->DataWrite();
    for (uint32_t t = 0; t < cfg.C; ++t) win[t] = (float)prompt[t];
    for (uint32_t i = 0; i < W; ++i) RunWindow(b);
    std::vector<double> times;
    for (uint32_t i = 0; i < K; ++i)
    {
        auto s = std::chrono::steady_clock::now();
        RunWindow(b);
        times.push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - s).count());
        // greedy feedback so the forwards are not identical (same cost either way)
        Mat* logits = b.model->GetOutput();
        const float* row = logits->DataRead() + (size_t)(cfg.C / 2) * cfg.V;
        uint32_t best = 0; float bv = row[0];
        for (uint32_t v = 1; v < cfg.V; ++v) if (row[v] > bv) { bv = row[v]; best = v; }
        win[cfg.C / 2 + 1] = (float)best;
    }
    double sum = 0; for (double t : times) sum += t;
    std::printf("{\"forwards\": %u, \"warmup\": %u, \"seconds_per_forward\": %.6f, \"build_seconds\": %.3f, "
                "\"threads\": %zu, \"times\": [", K, W, sum / K, build_s, GetGlobalThreadPool()->GetThreadCount());
    for (size_t i = 0; i < times.size(); ++i) std::printf("%s%.6f", i ? ", " : "", times[i]);
    std::printf("]}\n");
    return 0;
}

// Single generic operator from MatrixBase_Functions.h / MatrixBase_Mul.h on
// caller-supplied inputs.  --dims gives x,y,z per operand (colon separated).
static Dims3D ParseDims(const std::string& s)
{
    uint32_t x = 1, y = 1, z = 1;
    std::sscanf(s.c_str(), "%u,%u,%u", &x, &y, &z);
    return Dims3D(x, y, z);
}

static int ModeOp(const Args& a)
{
    Mgr& inst = Mgr::Instance();
    const std::string op = a.get("op");
    std::vector<Dims3D> dims;
    {
        std::string s = a.get("dims");
        size_t p = 0;
        while (p <= s.size())
        {
            size_t q = s.find(':', p);
            if (q == std::string::npos) q = s.size();
            dims.push_back(ParseDims(s.substr(p, q - p)));
            p = q + 1;
        }
    }
    // Operand 0 is the output; the rest are inputs read back to back from --in.
    std::vector<float> in = ReadF32(a.get("in"));
    std::vector<Mgr::MatrixRef> mats;
    size_t off = 0;
    for (size_t i = 0; i < dims.size(); ++i)
    {
        mats.push_back(inst.AllocateMatrix(dims[i], "op" + std::to_string(i)));
        const uint32_t n = mats.back()->GetElementCount();
        if (i == 0) { Fill(mats.back().get(), 0.0f); continue; }
        if (off + n > in.size()) { std::fprintf(stderr, "input too short\n"); return 2; }
        std::memcpy(mats.back()->DataWrite(), in.data() + off, n * 4);
        off += n;
    }
    auto M = [&](size_t i) { return mats[i].get(); };
    const float f = a.has("scalar") ? std::strtof(a.get("scalar").c_str(), nullptr) : 0.0f;
    std::vector<float> extra;
    if (op == "mul_none") Mul<TransposeMode::None>(M(0), M(1), M(2));
    else if (op == "mul_right") Mul<TransposeMode::Right>(M(0), M(1), M(2));
    else if (op == "matmul_strided_right")
    {
        // scores = Q_h K_h^T exactly as CausalSelfAttentionLayer.h:430-452 builds
        // it: head views of width --hd at column offset --off into [T x d]
        // operands 1 and 2, row stride d.
        const uint32_t hd = a.u("hd"), hoff = a.u("off"), T = M(1)->GetDimsY(), d = M(1)->GetDimsX();
        Mat qv; qv.SetData(M(1)->GetData(), hoff); qv.SetDims({hd, T});
        Mat kv; kv.SetData(M(2)->GetData(), hoff); kv.SetDims({hd, T});
        MatMul_Strided<TransposeMode::Right>(M(0), &qv, &kv, d, 1u, d, 1u, T, 1u);
    }
    else if (op == "matmul_strided_none")
    {
        // Y_h = P V_h into column block h of Y (CausalSelfAttentionLayer.h:478-497):
        // operand 0 is Y [T x d], operand 1 is P [T x T], operand 2 is V [T x d].
        const uint32_t hd = a.u("hd"), hoff = a.u("off"), T = M(1)->GetDimsY(), d = M(2)->GetDimsX();
        Mat vv; vv.SetData(M(2)->GetData(), hoff); vv.SetDims({hd, T});
        Mat yv; yv.SetData(M(0)->GetData(), hoff); yv.SetDims({hd, T});
        MatMul_Strided<TransposeMode::None>(&yv, M(1), &vv, T, 1u, d, 1u, d, 1u);
    }
    else if (op == "layernorm") LayerNormOp<T>(M(0), M(1), M(2), (MatrixBase<T>*)nullptr, (MatrixBase<T>*)nullptr, 1e-5f);
    else if (op == "layernorm_beta") LayerNormOp<T>(M(0), M(1), M(2), M(3), (MatrixBase<T>*)nullptr, 1e-5f);
    else if (op == "softmax") Softmax(M(0), M(1));
    else if (op == "gelu") GeluMat(M(0), M(1));
    else if (op == "add") Add(M(0), M(1), M(2));
    else if (op == "broadcast_add") BroadcastAdd(M(0), M(1), M(2));
    else if (op == "per_element_mul") PerElementMul(M(0), M(1), M(2));
    else if (op == "scale_add") ScaleAdd(M(0), M(1), M(2), M(3));
    else if (op == "scale") Scale(M(0), M(1), f);
    else if (op == "gather_rows") GatherRows(M(0), M(1), M(2));
    else if (op == "split_qkv")
    {
        // outputs q, k, v are operands 0..2; packed is operand 3
        Fill(M(1), 0.0f); Fill(M(2), 0.0f);
        SplitQKV(M(0), M(1), M(2), M(3));
        AppendMatrix(extra, M(1));
        AppendMatrix(extra, M(2));
    }
    else { std::fprintf(stderr, "unknown op %s\n", op.c_str()); return 2; }
    std::vector<float> out;
    AppendMatrix(out, M(0));
    out.insert(out.end(), extra.begin(), extra.end());
    WriteRaw(a.get("out"), out);
    return 0;
}

int main(int argc, char** argv)
{
    Tools::Logger::SetMinLevel(Tools::Logger::Level::Error);
    if (argc < 2) { std::fprintf(stderr, "usage: %s weights|greedy|forward|time|op|save|train [--key value]...\n", argv[0]); return 2; }
    const std::string mode = argv[1];
    Args a = ParseArgs(argc, argv, 2);
    if (mode == "greedy") return ModeGreedy(a);
    if (mode == "forward") return ModeForward(a);
    if (mode == "weights") return ModeWeights(a);
    if (mode == "save") return ModeSave(a);
    if (mode == "train") return ModeTrain(a);
    if (mode == "time") return ModeTime(a);
    if (mode == "op") return ModeOp(a);
    std::fprintf(stderr, "unknown mode %s\n", mode.c_str());
    return 2;
}
