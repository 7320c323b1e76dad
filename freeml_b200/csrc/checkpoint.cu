// FreeML checkpoints of a NanoLLM model, read straight into the decode engine.
//
// Format (written by Model::Save, ModelLibrary/Model.h:91-159, through
// SaveLoader, Loading/SaveLoader.h):
//   <dir>/model.guide            "LAYER <guid> <file>" per top-level layer,
//                                "INPUT_DIMS x y z", "OPTIMISER ...",
//                                "LOSSFUNC ..." (Model.h:343-379)
//   *.blob_layer  (text)         records "NAME k / DATA v / TYPE t [/ META m /
//                                GUID g]" closed by a ";" line; the first is
//                                the root (NAME Layer_Name, DATA <layer name>,
//                                TYPE ROOTLAYER_<type>); then sub-layers
//                                (TYPE LAYER_<type>, DATA <.blob_layer>),
//                                INT / UINT / FLOAT scalars (DATA <.blob_data>)
//                                and matrices (TYPE MATRIX, DATA <.blob_matrix>)
//                                (SaveLoader.h:499-577)
//   *.blob_matrix (text)         INTERNAL_NAME, GUID, DIMX, DIMY, DIMZ, DATA
//                                (SaveLoader.h:1523-1545)
//   *.blob_data   (binary)       raw little-endian payload (SaveLoader.h:1547-1563)
// The NanoLLM graph's layer names and blob keys (Examples/NanoLLM/NanoLLM.cpp:
// 268-348): embedding_token / embedding_pos (Embedding_Weights), block_<i>
// (TransformerBlock: LayerNorm0Data, AttentionLayerData {CSA_AttentionLayer,
// CSA_ProjLayer, NumHeads}, LayerNorm1Data, DenseFCData, DenseProjData;
// TransformerBlock.h:463-472, CausalSelfAttentionLayer.h:736-741), ln_f
// (GammaScale), lm_head (Dense_Weights, the token table's matrix: same GUID).
//
// Every weight matrix is stored in the layout the engine's packed order uses
// (canonical order: tok, pos, per layer {ln0, wqkv, wproj, ln1, wfc, wmlp},
// lnf), so packing is a concatenation of payloads after the shape checks.
// Host code only.
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "fml_common.cuh"

namespace fs = std::filesystem;

namespace fml {
namespace {

struct Record
{
    std::string name, data, type, meta, guid;
};

bool read_text(const fs::path& p, std::string& out)
{
    std::ifstream f(p, std::ios::binary);
    if (!f) return false;
    std::stringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

// "KEY value" lines; the value is everything after the first space.
void split_line(const std::string& line, std::string& key, std::string& value)
{
    std::string l = line;
    while (!l.empty() && (l.back() == '\r' || l.back() == '\n')) l.pop_back();
    const size_t sp = l.find(' ');
    key = sp == std::string::npos ? l : l.substr(0, sp);
    value = sp == std::string::npos ? std::string() : l.substr(sp + 1);
    while (!value.empty() && (value.back() == ' ' || value.back() == '\t')) value.pop_back();
}

int parse_records(const fs::path& p, std::vector<Record>& out)
{
    std::string text;
    if (!read_text(p, text)) return set_error(FML_ERR_INVALID, "checkpoint: cannot read %s", p.string().c_str());
    std::istringstream in(text);
    std::string line, key, value;
    Record cur;
    bool open = false;
    while (std::getline(in, line))
    {
        split_line(line, key, value);
        if (key == ";")
        {
            if (open) out.push_back(cur);
            cur = Record();
            open = false;
            continue;
        }
        if (key.empty()) continue;
        open = true;
        if (key == "NAME") cur.name = value;
        else if (key == "DATA") cur.data = value;
        else if (key == "TYPE") cur.type = value;
        else if (key == "META") cur.meta = value;
        else if (key == "GUID") cur.guid = value;
    }
    if (open) out.push_back(cur);
    return FML_OK;
}

struct LayerFile
{
    fs::path dir;
    std::string name, type;        // root record: layer name, ROOTLAYER_ / LAYER_ type
    std::map<std::string, Record> by_name;
};

int load_layer(const fs::path& p, LayerFile& lf)
{
    std::vector<Record> recs;
    FML_RC(parse_records(p, recs));
    lf.dir = p.parent_path();
    lf.by_name.clear();
    for (size_t i = 0; i < recs.size(); ++i)
    {
        if (i == 0 && recs[i].name == "Layer_Name")
        {
            lf.name = recs[i].data;
            lf.type = recs[i].type;
            continue;
        }
        lf.by_name[recs[i].name] = recs[i];
    }
    return FML_OK;
}

int sublayer(const LayerFile& parent, const char* key, LayerFile& out)
{
    auto it = parent.by_name.find(key);
    if (it == parent.by_name.end() || it->second.type.rfind("LAYER_", 0) != 0)
        return set_error(FML_ERR_INVALID, "checkpoint: layer %s has no sub-layer %s", parent.name.c_str(), key);
    FML_RC(load_layer(parent.dir / it->second.data, out));
    out.name = parent.name + "." + key;
    return FML_OK;
}

bool has_entry(const LayerFile& lf, const char* key) { return lf.by_name.count(key) != 0; }

int read_uint(const LayerFile& lf, const char* key, uint32_t& v)
{
    auto it = lf.by_name.find(key);
    if (it == lf.by_name.end() || it->second.type != "UINT")
        return set_error(FML_ERR_INVALID, "checkpoint: layer %s has no UINT %s", lf.name.c_str(), key);
    std::string raw;
    if (!read_text(lf.dir / it->second.data, raw) || raw.size() != sizeof(uint32_t))
        return set_error(FML_ERR_INVALID, "checkpoint: bad UINT payload %s of %s", key, lf.name.c_str());
    std::memcpy(&v, raw.data(), sizeof(v));
    return FML_OK;
}

struct Tensor
{
    fs::path data;  // .blob_data payload
    uint32_t x = 0, y = 0, z = 0;
    std::string guid, what;
};

int read_matrix(const LayerFile& lf, const char* key, Tensor& t)
{
    auto it = lf.by_name.find(key);
    if (it == lf.by_name.end() || it->second.type != "MATRIX")
        return set_error(FML_ERR_INVALID, "checkpoint: layer %s has no matrix %s", lf.name.c_str(), key);
    const fs::path hp = lf.dir / it->second.data;
    std::string text;
    if (!read_text(hp, text)) return set_error(FML_ERR_INVALID, "checkpoint: cannot read %s", hp.string().c_str());
    std::istringstream in(text);
    std::string line, k, v, data;
    bool hx = false, hy = false, hz = false;
    while (std::getline(in, line))
    {
        split_line(line, k, v);
        if (k == "DIMX") { t.x = (uint32_t)std::strtoul(v.c_str(), nullptr, 10); hx = true; }
        else if (k == "DIMY") { t.y = (uint32_t)std::strtoul(v.c_str(), nullptr, 10); hy = true; }
        else if (k == "DIMZ") { t.z = (uint32_t)std::strtoul(v.c_str(), nullptr, 10); hz = true; }
        else if (k == "GUID") t.guid = v;
        else if (k == "DATA") data = v;
    }
    if (!hx || !hy || !hz || data.empty())
        return set_error(FML_ERR_INVALID, "checkpoint: incomplete matrix header %s", hp.string().c_str());
    t.data = lf.dir / data;
    t.what = lf.name + "." + key;
    return FML_OK;
}

int expect_dims(const Tensor& t, uint32_t x, uint32_t y)
{
    if (t.x != x || t.y != y || t.z != 1u)
        return set_error(FML_ERR_INVALID, "checkpoint: %s is %u x %u x %u, expected %u x %u x 1", t.what.c_str(), t.x,
                         t.y, t.z, x, y);
    return FML_OK;
}

// The NanoLLM engine has no bias terms (NanoLLM.cpp:57, use_bias = false).
int expect_no_bias(const LayerFile& lf)
{
    if (has_entry(lf, "Dense_Bias") || has_entry(lf, "BetaShift"))
        return set_error(FML_ERR_UNSUPPORTED, "checkpoint: layer %s has a bias (the engine models use_bias = false)",
                         lf.name.c_str());
    return FML_OK;
}

int expect_transposed(const LayerFile& lf, uint32_t want)
{
    uint32_t v = 0;
    FML_RC(read_uint(lf, "Dense_Transposed", v));
    if (v != want)
        return set_error(FML_ERR_INVALID, "checkpoint: %s has Dense_Transposed = %u, expected %u", lf.name.c_str(), v,
                         want);
    return FML_OK;
}

// Locate every parameter of the checkpoint in canonical order and check the
// shapes; cfg gets V, C, d, H, L (max_batch 0).
int scan(const char* dir, fml_lm_config& cfg, std::vector<Tensor>& order)
{
    FML_REQUIRE(dir, "checkpoint: null directory");
    const fs::path root(dir);
    std::string guide;
    if (!read_text(root / "model.guide", guide))
        return set_error(FML_ERR_INVALID, "checkpoint: %s has no model.guide", dir);
    std::map<std::string, LayerFile> layers;  // by layer name
    {
        std::istringstream in(guide);
        std::string line, key, value;
        while (std::getline(in, line))
        {
            split_line(line, key, value);
            if (key != "LAYER") continue;
            const size_t sp = value.find(' ');
            if (sp == std::string::npos)
                return set_error(FML_ERR_INVALID, "checkpoint: bad model.guide line '%s'", line.c_str());
            LayerFile lf;
            FML_RC(load_layer(root / value.substr(sp + 1), lf));
            layers[lf.name] = lf;
        }
    }
    auto get = [&](const std::string& name, const char* type, LayerFile*& out) -> int {
        auto it = layers.find(name);
        if (it == layers.end()) return set_error(FML_ERR_INVALID, "checkpoint: no layer %s", name.c_str());
        if (it->second.type != std::string("ROOTLAYER_") + type)
            return set_error(FML_ERR_INVALID, "checkpoint: layer %s is %s, expected ROOTLAYER_%s", name.c_str(),
                             it->second.type.c_str(), type);
        out = &it->second;
        return FML_OK;
    };

    LayerFile *tok_l, *pos_l, *lnf_l, *head_l;
    FML_RC(get("embedding_token", "Embedding", tok_l));
    FML_RC(get("embedding_pos", "Embedding", pos_l));
    FML_RC(get("ln_f", "LayerNorm", lnf_l));
    FML_RC(get("lm_head", "Dense", head_l));
    Tensor tok, pos, lnf, head;
    FML_RC(read_matrix(*tok_l, "Embedding_Weights", tok));
    FML_RC(read_matrix(*pos_l, "Embedding_Weights", pos));
    const uint32_t d = tok.x, V = tok.y, C = pos.y;
    FML_RC(expect_dims(pos, d, C));
    uint32_t L = 0;
    while (layers.count("block_" + std::to_string(L))) ++L;
    if (L == 0) return set_error(FML_ERR_INVALID, "checkpoint: no block_0 layer");

    order.clear();
    order.push_back(tok);
    order.push_back(pos);
    uint32_t H = 0;
    for (uint32_t l = 0; l < L; ++l)
    {
        LayerFile* blk;
        FML_RC(get("block_" + std::to_string(l), "TransformerBlock", blk));
        LayerFile ln0, ln1, att, qkv_l, proj_l, fc_l, mlp_l;
        FML_RC(sublayer(*blk, "LayerNorm0Data", ln0));
        FML_RC(sublayer(*blk, "LayerNorm1Data", ln1));
        FML_RC(sublayer(*blk, "AttentionLayerData", att));
        FML_RC(sublayer(att, "CSA_AttentionLayer", qkv_l));
        FML_RC(sublayer(att, "CSA_ProjLayer", proj_l));
        FML_RC(sublayer(*blk, "DenseFCData", fc_l));
        FML_RC(sublayer(*blk, "DenseProjData", mlp_l));
        uint32_t h = 0;
        FML_RC(read_uint(att, "NumHeads", h));
        if (l == 0) H = h;
        else if (h != H) return set_error(FML_ERR_INVALID, "checkpoint: block_%u has %u heads, block_0 %u", l, h, H);
        for (LayerFile* lf : {&ln0, &ln1, &qkv_l, &proj_l, &fc_l, &mlp_l}) FML_RC(expect_no_bias(*lf));
        FML_RC(expect_transposed(qkv_l, 0));
        FML_RC(expect_transposed(proj_l, 1));
        FML_RC(expect_transposed(fc_l, 0));
        FML_RC(expect_transposed(mlp_l, 0));
        Tensor g0, wqkv, wproj, g1, wfc, wmlp;
        FML_RC(read_matrix(ln0, "GammaScale", g0));
        FML_RC(read_matrix(qkv_l, "Dense_Weights", wqkv));
        FML_RC(read_matrix(proj_l, "Dense_Weights", wproj));
        FML_RC(read_matrix(ln1, "GammaScale", g1));
        FML_RC(read_matrix(fc_l, "Dense_Weights", wfc));
        FML_RC(read_matrix(mlp_l, "Dense_Weights", wmlp));
        // Dims3D{x = cols, y = rows}: gamma one row of d; Dense W [in rows x
        // out cols], the attention projection stored [out x in] (Dense.h:34-36)
        FML_RC(expect_dims(g0, d, 1));
        FML_RC(expect_dims(wqkv, 3 * d, d));
        FML_RC(expect_dims(wproj, d, d));
        FML_RC(expect_dims(g1, d, 1));
        FML_RC(expect_dims(wfc, 4 * d, d));
        FML_RC(expect_dims(wmlp, d, 4 * d));
        for (const Tensor* t : {&g0, &wqkv, &wproj, &g1, &wfc, &wmlp}) order.push_back(*t);
    }
    FML_RC(expect_no_bias(*lnf_l));
    FML_RC(read_matrix(*lnf_l, "GammaScale", lnf));
    FML_RC(expect_dims(lnf, d, 1));
    order.push_back(lnf);
    // lm_head: the token table itself (tied, NanoLLM.cpp:333-345)
    FML_RC(expect_no_bias(*head_l));
    FML_RC(expect_transposed(*head_l, 1));
    FML_RC(read_matrix(*head_l, "Dense_Weights", head));
    if (head.guid.empty() || head.guid != tok.guid)
        return set_error(FML_ERR_UNSUPPORTED, "checkpoint: lm_head is not tied to the token embedding (GUID %s vs %s)",
                         head.guid.c_str(), tok.guid.c_str());
    if (H == 0 || d % H != 0) return set_error(FML_ERR_INVALID, "checkpoint: d_model %u, %u heads", d, H);
    cfg = fml_lm_config{V, C, d, H, L, 0};
    return FML_OK;
}

int read_payload(const Tensor& t, float* out)
{
    const uint64_t n = (uint64_t)t.x * t.y * t.z;
    std::ifstream f(t.data, std::ios::binary | std::ios::ate);
    if (!f) return set_error(FML_ERR_INVALID, "checkpoint: cannot read %s", t.data.string().c_str());
    const uint64_t bytes = (uint64_t)f.tellg();
    if (bytes != n * sizeof(float))
        return set_error(FML_ERR_INVALID, "checkpoint: %s payload is %llu bytes, expected %llu", t.what.c_str(),
                         (unsigned long long)bytes, (unsigned long long)(n * sizeof(float)));
    f.seekg(0);
    if (!f.read(reinterpret_cast<char*>(out), (std::streamsize)(n * sizeof(float))))
        return set_error(FML_ERR_INVALID, "checkpoint: short read of %s", t.data.string().c_str());
    return FML_OK;
}

int pack(const std::vector<Tensor>& order, float* out, uint64_t count)
{
    uint64_t off = 0;
    for (const Tensor& t : order)
    {
        const uint64_t n = (uint64_t)t.x * t.y * t.z;
        if (off + n > count) return set_error(FML_ERR_INVALID, "checkpoint: parameter buffer too small");
        FML_RC(read_payload(t, out + off));
        off += n;
    }
    if (off != count)
        return set_error(FML_ERR_INVALID, "checkpoint: %llu parameters, buffer holds %llu", (unsigned long long)off,
                         (unsigned long long)count);
    return FML_OK;
}

}  // namespace
}  // namespace fml

using namespace fml;

extern "C" {

int fml_checkpoint_config(const char* dir, fml_lm_config* cfg)
{
    FML_REQUIRE(cfg, "fml_checkpoint_config: null argument");
    std::vector<Tensor> order;
    fml_lm_config c{};
    FML_RC(scan(dir, c, order));
    *cfg = c;
    return FML_OK;
}

int fml_checkpoint_pack(const char* dir, float* params, uint64_t count)
{
    FML_REQUIRE(params || count == 0, "fml_checkpoint_pack: null buffer");
    std::vector<Tensor> order;
    fml_lm_config c{};
    FML_RC(scan(dir, c, order));
    return pack(order, params, count);
}

int fml_lm_load_checkpoint(fml_lm* lm, const char* dir, fml_stream_t stream)
{
    FML_REQUIRE(lm, "fml_lm_load_checkpoint: null engine");
    std::vector<Tensor> order;
    fml_lm_config c{};
    FML_RC(scan(dir, c, order));
    fml_lm_config mine{};
    FML_RC(fml_lm_get_config(lm, &mine));
    if (c.vocab != mine.vocab || c.context != mine.context || c.d_model != mine.d_model || c.n_head != mine.n_head ||
        c.n_layer != mine.n_layer)
        return set_error(FML_ERR_INVALID,
                         "fml_lm_load_checkpoint: checkpoint V%u C%u d%u H%u L%u, engine V%u C%u d%u H%u L%u", c.vocab,
                         c.context, c.d_model, c.n_head, c.n_layer, mine.vocab, mine.context, mine.d_model,
                         mine.n_head, mine.n_layer);
    const uint64_t n = fml_lm_param_count(&c);
    std::vector<float> host(n);
    FML_RC(pack(order, host.data(), n));
    return fml_lm_bind_packed(lm, host.data(), 1, stream);
}

}  // extern "C"
