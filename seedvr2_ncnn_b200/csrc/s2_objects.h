// Definitions of the opaque ABI objects (s2_context, s2_plan), shared by the
// library's translation units.
#pragma once

#include <map>
#include <memory>
#include <vector>

#include "s2_dist.h"
#include "s2_internal.h"

struct s2_plan
{
    s2::Plan plan;
    // attention schedule for the most recent text_lengths
    std::unique_ptr<s2::AttnSchedule> sched;
    std::vector<int> sched_text;
    int sched_device = -1;
};

struct s2_context
{
    s2::Context c;
    // Plans built from shapes inside s2_awa_forward, kept for later calls
    // (their device schedules must outlive the kernels that read them).
    std::map<std::vector<int>, std::unique_ptr<s2_plan>> plan_cache;
    // NCCL communicator of a multi-GPU job (s2_dist_init), or null.
    std::unique_ptr<s2::Dist> dist;
};

struct s2_shard
{
    s2::ShardPlan sp;
};

namespace s2 {
// Schedule of `plan` for these text lengths, rebuilt only when they change.
int ensure_schedule(s2_plan* p, const int* text_lengths, Context& ctx, const AttnSchedule** out);
} // namespace s2
