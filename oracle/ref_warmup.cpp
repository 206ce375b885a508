// TEST INFRASTRUCTURE ONLY -- linked beside the unmodified reference objects.
//
// The reference's NumaThreadPool has a start-up race: a worker thread reads
// the job generation counter only once it starts running
// (Int8-gemm/numa_threadpool.h:316 `my_gen = cb_->gen_.load()`), so a job
// dispatched before every worker has reached that line is never seen by the
// late workers and the dispatcher waits forever on `remaining_`
// (numa_threadpool.h:260-263).  It shows up on the first forward call when
// other threads (an OpenMP team) keep the cores busy.  ref_pool_warmup()
// creates the node-0 executor ahead of the first forward and gives its
// workers time to park on the futex, which closes that window.
#include <chrono>
#include <thread>
#include "numa_threadpool.h"

extern "C" void ref_pool_warmup(void) {
    static bool done = false;
    if (done) return;
    auto exec = nanovllm::NumaExecutorManager::get(0);
    (void)exec;
    std::this_thread::sleep_for(std::chrono::milliseconds(300));
    done = true;
}
