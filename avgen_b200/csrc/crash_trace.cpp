// Native backtraces on fatal signals, for diagnosing host crashes inside the
// extension (a segmentation fault in a launch path prints the C++ frames that
// led to it before Python's fault handler prints the Python stack).
//
// Opt-in: nothing is installed unless install_crash_backtrace() is called (the
// Python loader does so when AVGEN_NATIVE_BACKTRACE=1). The handler writes
// with write(2) and backtrace_symbols_fd only; backtrace() is primed once at
// install time so its first call (which may load libgcc) is not made inside
// the handler. After printing it hands the signal to the handler that was
// installed before it, then restores the default action and re-raises.
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstring>

namespace avgen {
namespace {

constexpr int kSignals[] = {SIGSEGV, SIGBUS, SIGFPE, SIGILL, SIGABRT};
struct sigaction g_prev[NSIG];
bool g_installed = false;

void write_text(const char* s) {
  ssize_t r = write(STDERR_FILENO, s, std::strlen(s));
  (void)r;
}

void on_fatal(int sig, siginfo_t* info, void* context) {
  write_text("avgen: fatal signal in native code; native backtrace:\n");
  void* frames[64];
  const int n = backtrace(frames, 64);
  backtrace_symbols_fd(frames, n, STDERR_FILENO);
  const struct sigaction& prev = g_prev[sig];
  if ((prev.sa_flags & SA_SIGINFO) != 0 && prev.sa_sigaction != nullptr) {
    prev.sa_sigaction(sig, info, context);
  } else if ((prev.sa_flags & SA_SIGINFO) == 0 && prev.sa_handler != SIG_DFL && prev.sa_handler != SIG_IGN &&
             prev.sa_handler != nullptr) {
    prev.sa_handler(sig);
  }
  signal(sig, SIG_DFL);
  raise(sig);
}

}  // namespace

bool install_crash_backtrace() {
  if (g_installed) return false;
  void* prime[4];
  (void)backtrace(prime, 4);
  for (int sig : kSignals) {
    struct sigaction sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.sa_sigaction = on_fatal;
    sigemptyset(&sa.sa_mask);
    sa.sa_flags = SA_SIGINFO;
    sigaction(sig, &sa, &g_prev[sig]);
  }
  g_installed = true;
  return true;
}

}  // namespace avgen
