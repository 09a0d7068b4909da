// plan_probe.cpp -- command-line probe of the screens' host-side planning
// (metal-flat_b200/csrc/cuda/plan.h) for the CPU test suite.  Reads one query
// per line on stdin and prints one result line:
//   chunks  n_qtiles n_tiles num_sms max_chunks min_chunks  -> n_chunks tiles_per_chunk
//   buffer  n_qtiles n_tiles num_sms tile_bytes              -> n_chunks tiles_per_chunk
//   large   n k m kp1 want lists_per_chunk num_sms budget    -> the LargePlan fields
#include <cstdio>
#include <cstring>
#include <iostream>
#include <sstream>
#include <string>

#include "plan.h"

int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        std::istringstream in(line);
        std::string op;
        in >> op;
        if (op == "chunks") {
            int nq, nt, sms, maxc, minc, nc = 0, tpc = 0;
            in >> nq >> nt >> sms >> maxc >> minc;
            mflat_cu::plan_chunks(nq, nt, sms, maxc, nc, tpc, minc);
            std::printf("%d %d\n", nc, tpc);
        } else if (op == "buffer") {
            int nq, nt, sms, nc = 0, tpc = 0;
            unsigned long long tb;
            in >> nq >> nt >> sms >> tb;
            mflat_cu::plan_buffer_chunks(nq, nt, sms, static_cast<size_t>(tb), nc, tpc);
            std::printf("%d %d\n", nc, tpc);
        } else if (op == "large") {
            long long n;
            int k, m, kp1, want, lpc, sms;
            unsigned long long budget;
            in >> n >> k >> m >> kp1 >> want >> lpc >> sms >> budget;
            const mflat_cu::LargePlan P =
                mflat_cu::plan_large(n, k, m, kp1, want, lpc, sms, static_cast<size_t>(budget));
            std::printf("%d %d %d %d %d %d %d %d %d %d %d %u %d\n", P.prepass ? 1 : 0,
                        P.two_stage ? 1 : 0, P.lists, P.stride_a, P.sample_a, P.stride_b,
                        P.sample_b, P.chunks_a, P.tpc_a, P.r_stat, P.r_guess, P.cap, P.batch);
        } else {
            std::printf("bad\n");
        }
        std::fflush(stdout);
    }
    return 0;
}
