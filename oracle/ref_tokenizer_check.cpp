// Test infrastructure, not product code: runs the reference engine's own tokenizer
// (model/qwen3tts/tokenizer.cpp with runtime/text/{bpe,unicode}.cpp, compiled from the
// reference tree by oracle/Makefile) on tokenizer files and a list of strings, so that the
// Python tokenizer's ids can be pinned to it (tests/golden/make_ref_golden.py).
//
//   ref_tokenizer_check VOCAB_JSON MERGES_TXT CONFIG_JSON CASES_JSON
//
// CASES_JSON is a JSON array of strings; the output is one line per string: the ids separated
// by spaces, then a tab, then the hex of the decoded UTF-8 bytes.
#include "model/qwen3tts/tokenizer.h"
#include "runtime/common/json.h"

#include <cstdio>
#include <fstream>
#include <sstream>
#include <string>

static std::string slurp(const char * path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) { std::fprintf(stderr, "cannot read %s\n", path); std::exit(2); }
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

int main(int argc, char ** argv) {
    if (argc != 5) { std::fprintf(stderr, "usage: %s vocab.json merges.txt config.json cases.json\n", argv[0]); return 2; }
    try {
        const std::string vocab = slurp(argv[1]), merges = slurp(argv[2]), cfg = slurp(argv[3]);
        const auto tok = navi::qwen3tts::Tokenizer::from_files(vocab, merges, cfg);
        const navi::Json cases = navi::Json::parse(slurp(argv[4]));
        for (const auto & c : cases.as_array()) {
            const auto ids = tok.encode(c.as_string());
            for (std::size_t i = 0; i < ids.size(); ++i) std::printf(i ? " %d" : "%d", ids[i]);
            std::printf("\t");
            for (unsigned char ch : tok.decode(ids)) std::printf("%02x", ch);
            std::printf("\n");
        }
        return 0;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
