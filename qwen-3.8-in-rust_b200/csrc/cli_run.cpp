// `qdec run`: the reference's `aqueduct run` (crates/cli/src/run.rs:254-420) over the C ABI of include/qdec.h and
// nothing else.  It loads a GGUF into HBM, feeds a prompt of raw ids, decodes greedily (or with the reference's
// sampler) plainly or with MTP speculative decoding (--spec k), prints the ids to stdout and the timings to
// stderr, and with --stats <file> writes one JSON object of the run's numbers.  The tokenizer, chat template,
// memory budget and disk tiers of the reference are outside this engine (its weights are resident in HBM).
//
//   qdec run --model <gguf> --ids 1,2,3 [--max-tokens 32] [--spec [k]] [--stats <file>] [--ids-only]
//            [--max-pos n] [--device d] [--gpus n] [--mode single|tp|replica]
//            [--temperature t] [--top-k k] [--top-p p] [--min-p m] [--seed s] [-v]
//
// --gpus n --mode tp: one sequence tensor-parallel over GPUs 0..n-1, one process per GPU (forked here; the
// ranks exchange their CUDA IPC handles over pipes) -- the ids are those of one GPU.  --mode replica: n
// independent copies of the run, one per GPU, and their aggregate tok/s.  Rank / replica 0 prints.
#include <sys/types.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cmath>
#include <csignal>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qdec.h"

namespace {

struct Args {
    std::string model;
    std::vector<uint32_t> ids;
    int max_tokens = 32;
    int spec = 0;
    std::string stats;
    bool ids_only = false;
    int max_pos = 0;
    int device = 0;
    int gpus = 1;
    std::string mode = "single";
    float temperature = 0.0f, top_p = 1.0f, min_p = 0.0f;
    int top_k = 0;
    uint64_t seed = 0;
    bool sampled = false;
    bool verbose = false;
};

constexpr int DEFAULT_SPEC_K = 3;  // `--spec` without a number (run.rs DEFAULT_SPEC_K)

[[noreturn]] void usage(const char* msg) {
    if (msg) fprintf(stderr, "qdec run: %s\n", msg);
    fprintf(stderr,
            "usage: qdec run --model <gguf> --ids <id,id,...> [--max-tokens n] [--spec [k]] [--stats <file>] [--ids-only]\n"
            "                [--max-pos n] [--device d] [--gpus n] [--mode single|tp|replica]\n"
            "                [--temperature t] [--top-k k] [--top-p p] [--min-p m] [--seed s] [-v]\n");
    exit(2);
}

bool parse_int(const char* s, long long& out) {
    char* end = nullptr;
    out = strtoll(s, &end, 10);
    return end && *end == '\0' && end != s;
}

Args parse(int argc, char** argv) {
    Args a;
    for (int i = 0; i < argc; i++) {
        const std::string k = argv[i];
        auto next = [&]() -> const char* {
            if (i + 1 >= argc) usage((k + " needs a value").c_str());
            return argv[++i];
        };
        long long v = 0;
        if (k == "--model") a.model = next();
        else if (k == "--ids") {
            std::string s = next();
            size_t p = 0;
            while (p <= s.size()) {
                size_t q = s.find(',', p);
                if (q == std::string::npos) q = s.size();
                std::string tok = s.substr(p, q - p);
                if (!tok.empty()) {
                    if (!parse_int(tok.c_str(), v) || v < 0 || v > 0xffffffffLL) usage(("--ids: bad id '" + tok + "'").c_str());
                    a.ids.push_back((uint32_t)v);
                }
                p = q + 1;
            }
        } else if (k == "--max-tokens") {
            if (!parse_int(next(), v) || v < 1) usage("--max-tokens: a positive integer");
            a.max_tokens = (int)v;
        } else if (k == "--spec") {
            // `--spec` alone takes the default k; `--spec k` a number (run.rs parse)
            if (i + 1 < argc && parse_int(argv[i + 1], v)) {
                if (v < 0 || v > 16) usage("--spec: 0..16");
                a.spec = (int)v;
                i++;
            } else {
                a.spec = DEFAULT_SPEC_K;
            }
        } else if (k == "--stats") a.stats = next();
        else if (k == "--ids-only") a.ids_only = true;
        else if (k == "--max-pos") {
            if (!parse_int(next(), v) || v < 1) usage("--max-pos: a positive integer");
            a.max_pos = (int)v;
        } else if (k == "--device") {
            if (!parse_int(next(), v) || v < 0) usage("--device: a device ordinal");
            a.device = (int)v;
        } else if (k == "--gpus") {
            if (!parse_int(next(), v) || v < 1 || v > 8) usage("--gpus: 1..8");
            a.gpus = (int)v;
        } else if (k == "--mode") {
            a.mode = next();
            if (a.mode != "single" && a.mode != "tp" && a.mode != "replica") usage("--mode: single, tp or replica");
        } else if (k == "--temperature") a.temperature = strtof(next(), nullptr), a.sampled = true;
        else if (k == "--top-k") {
            if (!parse_int(next(), v) || v < 0) usage("--top-k: >= 0");
            a.top_k = (int)v, a.sampled = true;
        } else if (k == "--top-p") a.top_p = strtof(next(), nullptr), a.sampled = true;
        else if (k == "--min-p") a.min_p = strtof(next(), nullptr), a.sampled = true;
        else if (k == "--seed") {
            if (!parse_int(next(), v) || v < 0) usage("--seed: >= 0");
            a.seed = (uint64_t)v, a.sampled = true;
        } else if (k == "-v" || k == "--verbose") a.verbose = true;
        else usage(("unknown argument " + k).c_str());
    }
    if (a.model.empty()) usage("--model is required");
    if (a.ids.empty()) usage("--ids is required (the prompt as raw token ids)");
    if (a.gpus > 1 && a.mode == "single") a.mode = "replica";
    if (a.gpus == 1) a.mode = "single";
    if (a.sampled && a.temperature == 0.0f) a.temperature = 1.0f;  // a sampler option alone samples at T = 1
    return a;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void check(int rc, const char* what) {
    if (rc != QDEC_OK) {
        fprintf(stderr, "qdec run: %s: %s\n", what, qdec_last_error());
        exit(1);
    }
}

std::string join(const std::vector<uint32_t>& v) {
    std::string s;
    for (size_t i = 0; i < v.size(); i++) s += (i ? "," : "") + std::to_string(v[i]);
    return s;
}

template <typename T>
std::string jlist(const std::vector<T>& v, const char* fmt) {
    std::string s = "[";
    char b[64];
    for (size_t i = 0; i < v.size(); i++) {
        snprintf(b, sizeof b, fmt, v[i]);
        s += (i ? "," : "") + std::string(b);
    }
    return s + "]";
}

// Ranks of a tensor-parallel run exchange their handles through the parent: rank r writes its handle to
// up[r], reads all of them from down[r]; after its last call it writes one byte to up[r] and waits for one on
// down[r] before freeing its state (no rank may unmap a block a peer still writes).
struct Pipes {
    int up[8][2], down[8][2];
};

bool read_full(int fd, void* p, size_t n) {
    uint8_t* b = (uint8_t*)p;
    while (n) {
        ssize_t r = read(fd, b, n);
        if (r <= 0) return false;
        b += r, n -= (size_t)r;
    }
    return true;
}
bool write_full(int fd, const void* p, size_t n) {
    const uint8_t* b = (const uint8_t*)p;
    while (n) {
        ssize_t r = write(fd, b, n);
        if (r <= 0) return false;
        b += r, n -= (size_t)r;
    }
    return true;
}

// One run (a rank of a TP group, a replica, or the only process): returns its exit status.
int run_one(const Args& a, int rank, int world, bool tp, Pipes* pp) {
    const bool lead = rank == 0;
    const int k = a.spec;
    const int n = (int)a.ids.size();
    const int max_pos = a.max_pos > 0 ? a.max_pos : n + a.max_tokens + k + 2;
    qdec_opts o{};
    o.device = tp || world > 1 ? rank : a.device;
    o.max_pos = max_pos + 64;
    qdec_model* m = nullptr;
    if (lead) fprintf(stderr, "loading %s on %s ...\n", a.model.c_str(), tp ? ("GPUs 0.." + std::to_string(world - 1) + " (tensor parallel)").c_str() : ("GPU " + std::to_string(o.device)).c_str());
    check(tp ? qdec_open_tp(a.model.c_str(), &o, rank, world, &m) : qdec_open(a.model.c_str(), &o, &m), "load");
    qdec_model_info info{};
    check(qdec_model_get_info(m, &info), "model info");
    if (lead)
        fprintf(stderr, "loaded in %.1f s: %u layers, %.3f GB of weights resident%s\n", info.load_secs, info.n_layer,
                info.weight_bytes / 1e9, tp ? " on this rank" : "");
    if (k > 0 && !info.has_mtp) {
        fprintf(stderr, "qdec run: --spec: this GGUF has no MTP block\n");
        return 1;
    }
    qdec_state* s = nullptr;
    check(qdec_state_new(m, k, max_pos, 32, &s), "state");
    if (tp) {
        uint8_t h[QDEC_TP_HANDLE_BYTES];
        check(qdec_tp_export(s, h), "tp export");
        std::vector<uint8_t> all((size_t)world * QDEC_TP_HANDLE_BYTES);
        if (!write_full(pp->up[rank][1], h, sizeof h) || !read_full(pp->down[rank][0], all.data(), all.size())) {
            fprintf(stderr, "qdec run: rank %d: handle exchange failed\n", rank);
            return 1;
        }
        check(qdec_tp_connect(s, all.data()), "tp connect");
    }
    if (a.sampled) check(qdec_set_sampler(s, a.temperature, a.top_k, a.top_p, a.min_p, a.seed), "sampler");
    if (lead)
        fprintf(stderr, "sampling: %s\n", a.sampled ? ("temperature " + std::to_string(a.temperature) + ", top_k " + std::to_string(a.top_k) +
                                                        ", top_p " + std::to_string(a.top_p) + ", min_p " + std::to_string(a.min_p) +
                                                        ", seed " + std::to_string(a.seed)).c_str()
                                                     : "greedy");
    // prefill (batched), then the plain loop or the speculative rounds (run.rs:300-383)
    const double t0 = now_s();
    uint32_t next = 0;
    check(k > 0 ? qdec_spec_prefill(s, a.ids.data(), n, &next) : qdec_prefill(s, a.ids.data(), n, &next), "prefill");
    const double prefill_s = now_s() - t0;
    if (lead) fprintf(stderr, "prefill (batched): %d tokens in %.3f s (%.1f tok/s)\n", n, prefill_s, n / prefill_s);
    std::vector<uint32_t> out;
    std::vector<double> step_secs;
    std::vector<int> round_accepted;
    int stopped = -1;
    const double t1 = now_s();
    if (k == 0) {
        for (;;) {
            if (qdec_is_stop(m, next)) {
                stopped = (int)next;
                break;
            }
            out.push_back(next);
            if ((int)out.size() >= a.max_tokens) break;
            const double ts = now_s();
            check(qdec_step(s, next, &next, nullptr), "step");
            step_secs.push_back(now_s() - ts);
            if (a.verbose && lead) fprintf(stderr, "  token %zu -> %u (%.4f s)\n", out.size(), next, step_secs.back());
        }
    } else {
        std::vector<uint32_t> em(k + 1);
        bool done = false;
        while (!done) {
            if (qdec_is_stop(m, next)) {
                stopped = (int)next;
                break;
            }
            out.push_back(next);
            if ((int)out.size() >= a.max_tokens) break;
            const double ts = now_s();
            int ne = 0;
            check(qdec_spec_round(s, next, em.data(), &ne), "spec round");
            step_secs.push_back(now_s() - ts);
            round_accepted.push_back(ne - 1);
            if (a.verbose && lead) fprintf(stderr, "  round %zu: accepted %d of %d (%.4f s)\n", round_accepted.size(), ne - 1, k, step_secs.back());
            for (int i = 0; i + 1 < ne && !done; i++) {
                if (qdec_is_stop(m, em[i])) {
                    stopped = (int)em[i];
                    done = true;
                } else {
                    out.push_back(em[i]);
                    if ((int)out.size() >= a.max_tokens) done = true;
                }
            }
            next = em[ne - 1];
        }
        if ((int)out.size() > a.max_tokens) out.resize(a.max_tokens);
    }
    const double decode_s = now_s() - t1;
    uint64_t c4[4] = {0, 0, 0, 0};
    if (k > 0) check(qdec_spec_counters(s, c4), "counters");
    if (tp) {  // every rank is past its last call before any rank frees its exchange block
        const uint8_t b = 1;
        uint8_t r = 0;
        if (!write_full(pp->up[rank][1], &b, 1) || !read_full(pp->down[rank][0], &r, 1)) return 1;
    }
    qdec_state_free(s);
    qdec_close(m);
    if (pp && !tp) {  // a replica reports its decode tokens and seconds for the aggregate
        const double r2[2] = {out.size() > 1 ? (double)(out.size() - 1) : 0.0, decode_s};
        if (!write_full(pp->up[rank][1], r2, sizeof r2)) return 1;
    }
    if (!lead) return 0;
    const int steps = std::max<int>(1, (int)step_secs.size());
    const double s_per_step = decode_s / steps;
    const double tok_s = out.size() > 1 ? (double)(out.size() - 1) / decode_s : 0.0;
    if (k == 0) {
        fprintf(stderr, "decode: %zu tokens, %.4f s/token (%.2f tok/s) = %.1f GB/s of weights%s\n", out.size(), s_per_step,
                1.0 / s_per_step, info.decode_bytes / s_per_step / 1e9,
                stopped >= 0 ? (", stopped at id " + std::to_string(stopped)).c_str() : "");
    } else {
        fprintf(stderr, "decode: %zu tokens, %.4f s/round, %.2f tok/s over %d rounds of --spec %d%s\n", out.size(), s_per_step, tok_s,
                (int)step_secs.size(), k, stopped >= 0 ? (", stopped at id " + std::to_string(stopped)).c_str() : "");
        fprintf(stderr, "spec: %llu rounds, %llu of %llu drafts accepted (%.1f %%), mean %.3f accepted per round, %.3f tokens per round\n",
                (unsigned long long)c4[0], (unsigned long long)c4[2], (unsigned long long)c4[1],
                c4[1] ? 100.0 * c4[2] / c4[1] : 0.0, c4[0] ? (double)c4[2] / c4[0] : 0.0, c4[0] ? (double)c4[3] / c4[0] : 0.0);
    }
    if (!a.stats.empty()) {
        FILE* f = fopen(a.stats.c_str(), "w");
        if (!f) {
            fprintf(stderr, "qdec run: write %s: %s\n", a.stats.c_str(), strerror(errno));
            return 1;
        }
        std::vector<int> hist(k + 1, 0);
        for (int r : round_accepted) hist[r]++;
        fprintf(f,
                "{\"model\":\"%s\",\"gpus\":%d,\"mode\":\"%s\",\"load_s\":%.3f,\"weight_bytes\":%llu,\"prompt_len\":%d,"
                "\"n_generated\":%zu,\"steps\":%d,\"prefill_s\":%.4f,\"decode_s\":%.4f,\"s_per_step\":%.5f,\"tok_s\":%.3f,"
                "\"step_secs\":%s,\"decode_bytes_per_token\":%llu,\"sampling\":\"%s\",\"seed\":%llu,\"spec_k\":%d",
                a.model.c_str(), world, tp ? "tp" : "single", info.load_secs, (unsigned long long)info.weight_bytes, n, out.size(),
                (int)step_secs.size(), prefill_s, decode_s, s_per_step, k > 0 ? tok_s : 1.0 / s_per_step,
                jlist(step_secs, "%.5f").c_str(), (unsigned long long)info.decode_bytes, a.sampled ? "sampled" : "greedy",
                (unsigned long long)a.seed, k);
        if (k > 0)
            fprintf(f, ",\"spec_rounds\":%llu,\"spec_drafted\":%llu,\"spec_accepted\":%llu,\"spec_emitted\":%llu,\"spec_hist\":%s,"
                       "\"spec_mean_accepted\":%.4f,\"spec_acceptance_rate\":%.4f,\"round_accepted\":%s",
                    (unsigned long long)c4[0], (unsigned long long)c4[1], (unsigned long long)c4[2], (unsigned long long)c4[3],
                    jlist(hist, "%d").c_str(), c4[0] ? (double)c4[2] / c4[0] : 0.0, c4[1] ? (double)c4[2] / c4[1] : 0.0,
                    jlist(round_accepted, "%d").c_str());
        fprintf(f, ",\"ids\":%s}\n", jlist(out, "%u").c_str());
        fclose(f);
    }
    if (a.ids_only) {
        printf("%s\n", join(out).c_str());
    } else {
        printf("prompt ids: %s\n", join(a.ids).c_str());
        printf("generated ids: %s\n", join(out).c_str());
    }
    fflush(stdout);
    return 0;
}

// Fork one process per GPU; for tensor parallelism relay the handles and the final barrier between them.
int run_forked(const Args& a) {
    const int world = a.gpus;
    const bool tp = a.mode == "tp";
    Pipes pp{};
    for (int r = 0; r < world; r++)
        if (pipe(pp.up[r]) || pipe(pp.down[r])) {
            perror("pipe");
            return 1;
        }
    std::vector<pid_t> pids;
    for (int r = 0; r < world; r++) {
        fflush(stdout);
        fflush(stderr);
        const pid_t p = fork();
        if (p < 0) {
            perror("fork");
            for (pid_t q : pids) kill(q, SIGTERM);
            return 1;
        }
        if (p == 0) {
            for (int q = 0; q < world; q++) {
                close(pp.up[q][0]);
                close(pp.down[q][1]);
            }
            _exit(run_one(a, r, world, tp, &pp));
        }
        pids.push_back(p);
    }
    for (int r = 0; r < world; r++) {
        close(pp.up[r][1]);
        close(pp.down[r][0]);
    }
    int status = 0;
    if (tp) {
        std::vector<uint8_t> all((size_t)world * QDEC_TP_HANDLE_BYTES);
        bool ok = true;
        for (int r = 0; r < world && ok; r++) ok = read_full(pp.up[r][0], all.data() + (size_t)r * QDEC_TP_HANDLE_BYTES, QDEC_TP_HANDLE_BYTES);
        for (int r = 0; r < world && ok; r++) ok = write_full(pp.down[r][1], all.data(), all.size());
        uint8_t b = 0;
        for (int r = 0; r < world && ok; r++) ok = read_full(pp.up[r][0], &b, 1);
        for (int r = 0; r < world && ok; r++) ok = write_full(pp.down[r][1], &b, 1);
        if (!ok) {  // a rank failed: stop the others (their device waits end on their own limits)
            for (pid_t q : pids) kill(q, SIGTERM);
            status = 1;
        }
    } else {  // replicas: the whole-box decode rate, every replica's tokens over the slowest replica's time
        double tokens = 0.0, slowest = 0.0, r2[2];
        bool ok = true;
        for (int r = 0; r < world && ok; r++) {
            ok = read_full(pp.up[r][0], r2, sizeof r2);
            if (ok) tokens += r2[0], slowest = std::max(slowest, r2[1]);
        }
        if (ok && slowest > 0) fprintf(stderr, "replicas: %d GPUs, %.0f tokens decoded, %.2f tok/s whole box\n", world, tokens, tokens / slowest);
        if (!ok) status = 1;
    }
    for (pid_t q : pids) {
        int st = 0;
        waitpid(q, &st, 0);
        if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) status = 1;
    }
    return status;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2 || std::string(argv[1]) != "run") usage(argc < 2 ? nullptr : ("unknown command " + std::string(argv[1])).c_str());
    const Args a = parse(argc - 2, argv + 2);
    if (a.gpus > 1) return run_forked(a);
    return run_one(a, 0, 1, false, nullptr);
}
