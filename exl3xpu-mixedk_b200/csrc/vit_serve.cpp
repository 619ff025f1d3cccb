// vit_serve.cpp -- exl3b_vit: the command-line worker over the C ABI.
//
// Drop-in for the reference's `viterbi_esimd` executable
// (quantize/viterbi_esimd.cpp:683-733 serve loop, :1005-1030 file mode), so the
// reference's "proc" transport (quantize.py:532-608) can drive the B200
// encoder unchanged:
//
//   exl3b_vit serve
//     Framed stdin/stdout worker.  stdout carries replies only; logs go to
//     stderr.  Request (48 bytes, little endian, struct "<IIiiQQ16s"):
//       u32 magic = 0x58545156, u32 op (0 quit, 1 run), i32 margin, i32 pivot,
//       u64 nseq, u64 xbytes, char code[16]
//     followed by xbytes of fp32 X [nseq][256].  Reply (16 bytes, "<IiQ"):
//       u32 magic, i32 rc, u64 nbytes, then nbytes of int32 states (rc == 0).
//     rc 7 answers a malformed run request (op not 0/1, xbytes != nseq*256*4,
//     nseq > 2^22) and the worker keeps serving; a bad magic or a short X
//     read ends the worker with exit status 1; EOF or op 0 ends it with 0.
//     Other rc values are xtq_vit_run's (0 ok, 1 no device, 2 alloc, 4 device
//     error, 5 over XTQ_VIT_MAXBYTES, 6 nseq out of range, 7 bad request).
//     The device is XTQ_VIT_DEVIDX (set by the spawner), like the
//     reference's per-child device selector.
//
//   exl3b_vit X.bin nseq code margin pivot states.bin [iters]
//     File mode: X.bin = nseq*256 fp32, states.bin = nseq*256 int32; with
//     iters > 1 the call is repeated and the mean time per call is logged.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "exl3b200.h"

namespace {

constexpr uint32_t kMagic = 0x58545156u;
constexpr uint64_t kMaxSeq = 1ull << 22;

#pragma pack(push, 1)
struct Request {
    uint32_t magic;
    uint32_t op;
    int32_t margin;
    int32_t pivot;
    uint64_t nseq;
    uint64_t xbytes;
    char code[16];
};
struct Reply {
    uint32_t magic;
    int32_t rc;
    uint64_t nbytes;
};
#pragma pack(pop)
static_assert(sizeof(Request) == 48, "request frame is 48 bytes");
static_assert(sizeof(Reply) == 16, "reply frame is 16 bytes");

bool read_all(void* dst, size_t bytes) {
    return bytes == 0 || fread(dst, 1, bytes, stdin) == bytes;
}

void reply(int rc, const void* data, uint64_t nbytes) {
    const Reply r{kMagic, rc, nbytes};
    fwrite(&r, sizeof(r), 1, stdout);
    if (nbytes) fwrite(data, 1, nbytes, stdout);
    fflush(stdout);
}

int serve() {
    std::vector<float> x;
    std::vector<int32_t> states;
    for (;;) {
        Request q;
        const size_t got = fread(&q, 1, sizeof(q), stdin);
        if (got == 0) return 0;                        // EOF: caller is done
        if (got != sizeof(q)) {
            fprintf(stderr, "exl3b_vit serve: request frame truncated after %zu of 48 bytes\n", got);
            return 1;
        }
        q.code[15] = 0;
        if (q.magic != kMagic) {
            fprintf(stderr, "exl3b_vit serve: frame magic 0x%08x is not 0x58545156; closing\n", q.magic);
            return 1;
        }
        if (q.op == 0) return 0;
        if (q.op != 1 || q.nseq > kMaxSeq || q.xbytes != q.nseq * 256ull * 4ull) {
            reply(7, nullptr, 0);
            continue;
        }
        x.resize((size_t)q.nseq * 256);
        if (!read_all(x.data(), (size_t)q.xbytes)) {
            fprintf(stderr, "exl3b_vit serve: stream ended inside the request's target block\n");
            return 1;
        }
        states.resize((size_t)q.nseq * 256);
        const int rc = xtq_vit_run(x.data(), (int)q.nseq, q.code, q.margin, q.pivot,
                                   states.data());
        if (rc) {
            fprintf(stderr, "exl3b_vit serve: rc=%d: %s\n", rc, exl3b_last_error());
            reply(rc, nullptr, 0);
        } else {
            reply(0, states.data(), (uint64_t)states.size() * 4);
        }
    }
}

int file_mode(int argc, char** argv) {
    const char* xfile = argv[1];
    const long nseq = strtol(argv[2], nullptr, 10);
    const char* code = argv[3];
    const int margin = atoi(argv[4]);
    const int pivot = atoi(argv[5]);
    const char* sfile = argv[6];
    const int iters = argc > 7 ? atoi(argv[7]) : 1;
    if (nseq <= 0 || nseq > (long)kMaxSeq || iters < 1) {
        fprintf(stderr, "exl3b_vit: bad nseq / iters\n");
        return 2;
    }
    std::vector<float> x((size_t)nseq * 256);
    FILE* f = fopen(xfile, "rb");
    if (!f || fread(x.data(), 4, x.size(), f) != x.size()) {
        fprintf(stderr, "exl3b_vit: cannot read %ld sequences from %s\n", nseq, xfile);
        if (f) fclose(f);
        return 2;
    }
    fclose(f);
    std::vector<int32_t> st(x.size());
    int rc = 0;
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < iters && !rc; ++i)
        rc = xtq_vit_run(x.data(), (int)nseq, code, margin, pivot, st.data());
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (rc) {
        fprintf(stderr, "exl3b_vit: rc=%d: %s\n", rc, exl3b_last_error());
        return rc;
    }
    fprintf(stderr, "exl3b_vit: %ld seqs x %d calls, %.3f ms/call, %.2f M weights/s\n", nseq,
            iters, 1e3 * s / iters, nseq * 256.0 * iters / s / 1e6);
    FILE* o = fopen(sfile, "wb");
    if (!o || fwrite(st.data(), 4, st.size(), o) != st.size()) {
        fprintf(stderr, "exl3b_vit: cannot write %s\n", sfile);
        if (o) fclose(o);
        return 2;
    }
    fclose(o);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && strcmp(argv[1], "serve") == 0) return serve();
    if (argc < 7) {
        fprintf(stderr,
                "usage: %s serve\n"
                "       %s X.bin nseq code[mul1|mul1p|mul1t] margin pivot states.bin [iters]\n",
                argv[0], argv[0]);
        return 1;
    }
    return file_mode(argc, argv);
}
