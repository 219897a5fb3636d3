// st_check.cpp — drives the drop-in SentenceTransformer the way the reference's CLI and
// server do (construct from a model directory, encode / encode_batch), for the
// model-level test in tests/test_dropin_gpu.py.
//
//   st_check <model_dir> <texts_file> <out_prefix>
// reads one text per line and writes, as float32 [rows, dim] unless noted:
//   <out_prefix>.ids         per text: int32 count, then the ids;
//   <out_prefix>.batch       encode_batch of the texts;
//   <out_prefix>.big         encode_batch of the texts repeated 40 times (tokenised on
//                            several host threads);
//   <out_prefix>.single      encode, one text at a time;
//   <out_prefix>.concurrent  encode from eight threads sharing the object at once, as the
//                            reference's HTTP server does (merged into shared device batches).
//   st_check <model_dir> <ids_file> <out_prefix> ids
// reads token ids in the .ids format and writes <out_prefix>.batch from encode_ids (the
// path of models whose tokenizer this build does not include, e.g. bge-m3).
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "sentence_transformers.h"

int main(int argc, char **argv)
{
    if (argc != 4 && !(argc == 5 && std::string(argv[4]) == "ids")) {
        std::fprintf(stderr, "usage: st_check <model_dir> <texts_file> <out_prefix> [ids]\n");
        return 2;
    }
    try {
        SentenceTransformer model(argv[1]);
        if (argc == 5) {
            std::ifstream in(argv[2], std::ios::binary);
            std::vector<std::vector<int32_t>> seqs;
            for (int32_t n = 0; in.read(reinterpret_cast<char *>(&n), 4);) {
                std::vector<int32_t> v(n);
                in.read(reinterpret_cast<char *>(v.data()), 4 * n);
                seqs.push_back(v);
            }
            std::ofstream batch(std::string(argv[3]) + ".batch", std::ios::binary);
            for (const auto &e : model.encode_ids(seqs))
                batch.write(reinterpret_cast<const char *>(e.data()), 4 * e.size());
            bool threw = false;  // text needs the SentencePiece tokenizer, absent from this build
            try {
                (void)model.tokenize("text");
            } catch (const std::exception &) {
                threw = true;
            }
            std::printf("dim %zu, %zu id sequences, text rejected %d\n", model.get_embedding_dimension(), seqs.size(),
                        threw ? 1 : 0);
            return 0;
        }
        std::vector<std::string> texts;
        std::ifstream in(argv[2]);
        for (std::string line; std::getline(in, line);) texts.push_back(line);
        const std::string pre = argv[3];
        std::ofstream ids(pre + ".ids", std::ios::binary), batch(pre + ".batch", std::ios::binary),
            single(pre + ".single", std::ios::binary);
        for (const auto &t : texts) {
            const std::vector<int32_t> v = model.tokenize(t);
            const int32_t n = static_cast<int32_t>(v.size());
            ids.write(reinterpret_cast<const char *>(&n), 4);
            ids.write(reinterpret_cast<const char *>(v.data()), 4 * n);
        }
        for (const auto &e : model.encode_batch(texts))
            batch.write(reinterpret_cast<const char *>(e.data()), 4 * e.size());
        {
            // a batch large enough to be tokenised on several host threads: the texts 40 times
            std::vector<std::string> big;
            for (int r = 0; r < 40; ++r) big.insert(big.end(), texts.begin(), texts.end());
            std::ofstream out(pre + ".big", std::ios::binary);
            for (const auto &e : model.encode_batch(big)) out.write(reinterpret_cast<const char *>(e.data()), 4 * e.size());
        }
        for (const auto &t : texts) {
            const std::vector<float> e = model.encode(t);
            single.write(reinterpret_cast<const char *>(e.data()), 4 * e.size());
        }
        std::vector<std::vector<float>> conc(texts.size());
        std::vector<std::string> errs(8);
        {
            std::vector<std::thread> pool;
            for (int t = 0; t < 8; ++t)
                pool.emplace_back([&, t] {
                    try {
                        for (int rep = 0; rep < 4; ++rep)  // several rounds, so that calls overlap
                            for (size_t i = t; i < texts.size(); i += 8) conc[i] = model.encode(texts[i]);
                    } catch (const std::exception &ex) {
                        errs[t] = ex.what();
                    }
                });
            for (auto &th : pool) th.join();
        }
        for (const auto &e : errs)
            if (!e.empty()) throw std::runtime_error("concurrent encode: " + e);
        std::ofstream concurrent(pre + ".concurrent", std::ios::binary);
        for (const auto &e : conc) concurrent.write(reinterpret_cast<const char *>(e.data()), 4 * e.size());
        std::printf("dim %zu, %zu texts\n", model.get_embedding_dimension(), texts.size());
    } catch (const std::exception &ex) {
        std::fprintf(stderr, "error: %s\n", ex.what());
        return 1;
    }
    return 0;
}
