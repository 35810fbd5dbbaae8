// bccl_run: starts N ranks of a program on this machine, without MPI.
//
//   bccl_run -np 4 [--timeout SEC] [--id-file PATH] [--gpus] -- ./program args...
//   bccl_run -np 8 --nnodes 2 --node-rank K --master ADDR:PORT [--gpus] -- ./program args...
//   bccl_run -np 4 --tag-output -- ./program      # every output line prefixed with "[rank R] "
//
// Multi-node (one bccl_run per node, like torchrun): node K runs global ranks K*np .. K*np+np-1
// of nnodes*np; BCCL_MASTER=ADDR:PORT is exported instead of an id file, and global rank 0
// (on node 0, whose address ADDR must be) listens on PORT for the bootstrap.
//
// Each child gets BCCL_RANK, BCCL_WORLD_SIZE, BCCL_LOCAL_RANK, BCCL_LOCAL_SIZE and BCCL_ID_FILE
// (a fresh path in a private temp directory unless --id-file is given). Rank 0 creates the unique
// id with Communicator::GetUniqueId and writes "ip:port" to that file (write to PATH.tmp, then
// rename); the others wait for it. With --gpus, BCCL_DEVICE=<local rank> is exported too.
// The launcher forwards SIGINT/SIGTERM to every child, and when one child fails (non-zero exit
// or a signal) or the timeout expires it terminates the others (SIGTERM, then SIGKILL after 5 s)
// and exits with the first failure's code. All children run in one process group of their own.
//
// Parity: the reference's tests are launched by `mpirun -np N` and broadcast the unique id with
// MPI_Bcast (OriginCCL tests/test_common.cpp:465-477); MPI is not part of this library.
#include <poll.h>
#include <signal.h>
#include <sys/stat.h>
#include <sys/types.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

volatile sig_atomic_t g_signal = 0;

void OnSignal(int sig) { g_signal = sig; }

int Usage() {
    std::fprintf(stderr,
                 "usage: bccl_run -np N [--timeout SEC] [--id-file PATH] [--gpus] [--tag-output]\n"
                 "                [--nnodes M --node-rank K --master ADDR:PORT] -- program [args...]\n");
    return 2;
}

// One forwarded stream of one rank (--tag-output).
struct Tagger {
    int fd;               // read end of the rank's pipe, -1 once closed
    int out;              // where the prefixed lines go
    std::string prefix;
    std::string partial;  // an incomplete last line
};

// Forwards whatever the ranks wrote, line by line with their prefix, until no pipe has data
// for wait_ms (0: until nothing is ready now) or every pipe has closed.
void PumpTaggers(std::vector<Tagger>* taggers, int wait_ms) {
    for (;;) {
        std::vector<pollfd> pf;
        std::vector<size_t> idx;
        for (size_t i = 0; i < taggers->size(); ++i) {
            if ((*taggers)[i].fd >= 0) {
                pf.push_back({(*taggers)[i].fd, POLLIN, 0});
                idx.push_back(i);
            }
        }
        if (pf.empty() || poll(pf.data(), pf.size(), wait_ms) <= 0) return;
        for (size_t k = 0; k < pf.size(); ++k) {
            if (!pf[k].revents) continue;
            Tagger& t = (*taggers)[idx[k]];
            char buf[4096];
            const ssize_t n = read(t.fd, buf, sizeof(buf));
            if (n <= 0) {
                close(t.fd);
                t.fd = -1;
                continue;
            }
            t.partial.append(buf, static_cast<size_t>(n));
            size_t nl;
            while ((nl = t.partial.find('\n')) != std::string::npos) {
                const std::string line = t.prefix + t.partial.substr(0, nl + 1);
                (void)!write(t.out, line.data(), line.size());
                t.partial.erase(0, nl + 1);
            }
        }
    }
}

// Signals the ranks' process group (which also reaches the ranks' own children), then any
// rank that is not done in case it moved to another group.
void KillAll(pid_t group, const std::vector<pid_t>& pids, const std::vector<bool>& done, int sig) {
    if (group > 0) kill(-group, sig);
    for (size_t i = 0; i < pids.size(); ++i)
        if (!done[i]) kill(pids[i], sig);
}

}  // namespace

int main(int argc, char** argv) {
    int np = 0, nnodes = 1, node_rank = 0;
    double timeout_s = 0;
    bool gpus = false, tag = false;
    std::string id_file, master;
    int i = 1;
    for (; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--") {
            ++i;
            break;
        }
        if ((a == "-np" || a == "-n") && i + 1 < argc) {
            np = std::atoi(argv[++i]);
        } else if (a == "--timeout" && i + 1 < argc) {
            timeout_s = std::atof(argv[++i]);
        } else if (a == "--id-file" && i + 1 < argc) {
            id_file = argv[++i];
        } else if (a == "--gpus") {
            gpus = true;
        } else if (a == "--tag-output") {
            tag = true;
        } else if (a == "--nnodes" && i + 1 < argc) {
            nnodes = std::atoi(argv[++i]);
        } else if (a == "--node-rank" && i + 1 < argc) {
            node_rank = std::atoi(argv[++i]);
        } else if (a == "--master" && i + 1 < argc) {
            master = argv[++i];
        } else if (a[0] != '-') {
            break;  // program without a "--" separator
        } else {
            return Usage();
        }
    }
    if (np < 1 || i >= argc || nnodes < 1 || node_rank < 0 || node_rank >= nnodes) return Usage();
    if (nnodes > 1 && master.find(':') == std::string::npos) {
        std::fprintf(stderr, "bccl_run: --nnodes > 1 needs --master ADDR:PORT\n");
        return 2;
    }
    char** prog = argv + i;

    std::string tmpdir;
    if (!master.empty()) {
        // no id file: the ranks find rank 0 at the master address
    } else if (id_file.empty()) {
        char tmpl[] = "/tmp/bccl_run.XXXXXX";
        if (mkdtemp(tmpl) == nullptr) {
            std::perror("bccl_run: mkdtemp");
            return 1;
        }
        tmpdir = tmpl;
        id_file = tmpdir + "/unique_id";
    } else {
        unlink(id_file.c_str());
    }

    struct sigaction sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.sa_handler = OnSignal;
    sigaction(SIGINT, &sa, nullptr);
    sigaction(SIGTERM, &sa, nullptr);

    std::vector<pid_t> pids(np, -1);
    // --tag-output: each rank's stdout / stderr through a pipe, forwarded line by line with a
    // "[rank R] " prefix (global rank).
    std::vector<Tagger> taggers;
    pid_t group = 0;
    for (int r = 0; r < np; ++r) {
        int out_pipe[2] = {-1, -1}, err_pipe[2] = {-1, -1};
        if (tag && (pipe(out_pipe) != 0 || pipe(err_pipe) != 0)) {
            std::perror("bccl_run: pipe");
            return 1;
        }
        pid_t pid = fork();
        if (pid < 0) {
            std::perror("bccl_run: fork");
            return 1;
        }
        if (pid == 0) {
            if (tag) {
                dup2(out_pipe[1], STDOUT_FILENO);
                dup2(err_pipe[1], STDERR_FILENO);
                close(out_pipe[0]);
                close(out_pipe[1]);
                close(err_pipe[0]);
                close(err_pipe[1]);
            }
            setpgid(0, group);
            setenv("BCCL_RANK", std::to_string(node_rank * np + r).c_str(), 1);
            setenv("BCCL_WORLD_SIZE", std::to_string(nnodes * np).c_str(), 1);
            setenv("BCCL_LOCAL_RANK", std::to_string(r).c_str(), 1);
            setenv("BCCL_LOCAL_SIZE", std::to_string(np).c_str(), 1);
            if (!master.empty()) {
                setenv("BCCL_MASTER", master.c_str(), 1);
            } else {
                setenv("BCCL_ID_FILE", id_file.c_str(), 1);
            }
            if (gpus) setenv("BCCL_DEVICE", std::to_string(r).c_str(), 1);
            execvp(prog[0], prog);
            std::fprintf(stderr, "bccl_run: exec %s: %s\n", prog[0], std::strerror(errno));
            _exit(127);
        }
        if (group == 0) group = pid;
        setpgid(pid, group);
        pids[r] = pid;
        if (tag) {
            close(out_pipe[1]);
            close(err_pipe[1]);
            const std::string prefix = "[rank " + std::to_string(node_rank * np + r) + "] ";
            taggers.push_back({out_pipe[0], STDOUT_FILENO, prefix, {}});
            taggers.push_back({err_pipe[0], STDERR_FILENO, prefix, {}});
        }
    }

    std::vector<bool> done(np, false);
    int remaining = np, first_fail = 0;
    bool terminating = false;
    auto t0 = std::chrono::steady_clock::now();
    auto term_at = t0;
    bool killed = false;
    while (remaining > 0) {
        PumpTaggers(&taggers, 0);
        int status = 0;
        pid_t pid = waitpid(-1, &status, WNOHANG);
        if (pid > 0) {
            for (int r = 0; r < np; ++r) {
                if (pids[r] != pid) continue;
                done[r] = true;
                --remaining;
                int code = WIFEXITED(status) ? WEXITSTATUS(status) : 128 + WTERMSIG(status);
                if (code != 0 && first_fail == 0 && !terminating) {
                    first_fail = code;
                    std::fprintf(stderr, "bccl_run: rank %d exited with %d; stopping the others\n", r, code);
                }
            }
            continue;
        }
        const double elapsed = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (!terminating && (first_fail != 0 || g_signal != 0 || (timeout_s > 0 && elapsed > timeout_s))) {
            if (first_fail == 0) {
                first_fail = g_signal != 0 ? 128 + g_signal : 124;
                std::fprintf(stderr, "bccl_run: %s; stopping all ranks\n", g_signal ? "signal" : "timeout");
            }
            terminating = true;
            term_at = std::chrono::steady_clock::now();
            KillAll(group, pids, done, SIGTERM);
        }
        if (terminating && !killed && std::chrono::steady_clock::now() - term_at > std::chrono::seconds(5)) {
            KillAll(group, pids, done, SIGKILL);
            killed = true;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    if (terminating || first_fail != 0) kill(-group, SIGKILL);  // leftovers of failed ranks
    PumpTaggers(&taggers, 200);  // what the ranks wrote last (their pipes close as they exit)
    for (Tagger& t : taggers) {
        if (!t.partial.empty()) {
            const std::string line = t.prefix + t.partial + "\n";
            (void)!write(t.out, line.data(), line.size());
        }
        if (t.fd >= 0) close(t.fd);
    }
    if (!tmpdir.empty()) {
        unlink(id_file.c_str());
        unlink((id_file + ".tmp").c_str());
        rmdir(tmpdir.c_str());
    }
    return first_fail;
}
