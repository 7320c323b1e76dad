// Test infrastructure: runs the reference's own NanoLLM character-vocabulary
// code (Examples/NanoLLM/NanoLLM.cpp:95-206: Vocab, BuildVocab, encode,
// decode, DecodeMatrixTokens) by compiling that example source here with its
// main() renamed.  Compiled by oracle/Makefile into oracle/_ref/; nothing in
// the product links or runs it.
//
//   ref_vocab CORPUS TEXT IDS OUTDIR
//     CORPUS  bytes the vocabulary is built from (BuildVocab)
//     TEXT    bytes to encode with the built map (encode)
//     IDS     little-endian uint32 ids to decode (decode, DecodeMatrixTokens)
//   writes OUTDIR/{unique.bin, corpus_ids.bin, encode.bin, decode.bin,
//   decode_tokens.bin}
#define main nanollm_example_main
#include <Examples/NanoLLM/NanoLLM.cpp>
#undef main

static std::vector<char> ReadBytes(const std::string& p)
{
    std::ifstream f(p, std::ios::binary);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

template <class V>
static void WriteBytes(const std::string& p, const V& v)
{
    std::ofstream f(p, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(v[0])));
}

int main(int argc, char** argv)
{
    if (argc != 5)
    {
        std::fprintf(stderr, "usage: %s CORPUS TEXT IDS OUTDIR\n", argv[0]);
        return 2;
    }
    const std::string out = argv[4];
    Vocab vocab = BuildVocab(ReadBytes(argv[1]));
    const std::vector<char> text = ReadBytes(argv[2]);
    const std::vector<char> idb = ReadBytes(argv[3]);
    std::vector<uint32_t> ids(idb.size() / 4);
    std::memcpy(ids.data(), idb.data(), ids.size() * 4);

    WriteBytes(out + "/unique.bin", vocab.unique);
    WriteBytes(out + "/corpus_ids.bin", vocab.ids);
    WriteBytes(out + "/encode.bin", encode(std::string(text.begin(), text.end()), vocab.toId));
    WriteBytes(out + "/decode.bin", decode(ids, vocab.toChar));

    // DecodeMatrixTokens on a one-column matrix of ids (token ids as floats)
    auto& inst = MatrixManager<float, MatType>::Instance();
    auto m = inst.AllocateMatrix({1u, (uint32_t)ids.size(), 1u}, "ids");
    for (uint32_t t = 0; t < ids.size(); ++t) m->SetValue(0u, t, 0u, (float)ids[t]);
    const std::string dt = DecodeMatrixTokens(m.get(), vocab.unique);
    WriteBytes(out + "/decode_tokens.bin", dt);
    return 0;
}
