// Drives mg::watch_wait (metalgym_b200/csrc/watchdog.h) with fake streams,
// communicators and clocks; prints one line per scenario:
//   <name> <result> <drained> <aborts> <polls> <released first>
#include <cstdio>

#include "watchdog.h"

namespace {

struct Fake {
    int finishAtPoll = -1;      // done() returns 1 from this poll on (-1: never on its own)
    int peerErrorAtPoll = -1;   // peerError() returns 1 from this poll on
    int cudaErrorAtPoll = -1;   // done() returns -1 at this poll
    bool drainsAfterAbort = true;
    int polls = 0, aborts = 0, releases = 0;
    bool abortBeforeRelease = false;  // NCCL's abort would wait for good on a live graph
    double clock = 0.0;         // advances 0.001 s per pause
};

int done(void* p) {
    Fake* f = static_cast<Fake*>(p);
    const int k = f->polls++;
    if (f->cudaErrorAtPoll >= 0 && k >= f->cudaErrorAtPoll) return -1;
    if (f->aborts > 0) return f->drainsAfterAbort ? 1 : 0;
    return f->finishAtPoll >= 0 && k >= f->finishAtPoll ? 1 : 0;
}
int peer(void* p) {
    Fake* f = static_cast<Fake*>(p);
    return f->peerErrorAtPoll >= 0 && f->polls > f->peerErrorAtPoll ? 1 : 0;
}
void release(void* p) { static_cast<Fake*>(p)->releases++; }
void abort_(void* p) {
    Fake* f = static_cast<Fake*>(p);
    if (f->releases == 0) f->abortBeforeRelease = true;
    f->aborts++;
}
double now(void* p) { return static_cast<Fake*>(p)->clock; }
void pause_(void* p) { static_cast<Fake*>(p)->clock += 0.001; }

void run(const char* name, Fake f, double limit, double drain) {
    mg::WatchOps o{&f, done, peer, release, abort_, now, pause_};
    bool drained = false;
    const int r = mg::watch_wait(o, limit, drain, &drained);
    std::printf("%s %d %d %d %d %d\n", name, r, drained ? 1 : 0, f.aborts, f.polls,
                f.aborts > 0 && !f.abortBeforeRelease ? 1 : 0);
}

}  // namespace

int main() {
    Fake finishes;
    finishes.finishAtPoll = 50;
    run("finishes", finishes, 1.0, 1.0);
    Fake peer_error;
    peer_error.peerErrorAtPoll = 20;
    run("peer_error", peer_error, 1.0, 1.0);
    Fake hangs;
    run("timeout", hangs, 0.1, 1.0);
    Fake stuck;
    stuck.drainsAfterAbort = false;
    run("timeout_undrained", stuck, 0.1, 0.05);
    Fake cuda_error;
    cuda_error.cudaErrorAtPoll = 7;
    run("cuda_error", cuda_error, 1.0, 1.0);
    return 0;
}
