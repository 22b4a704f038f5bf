"""Golden greedy token streams from the REFERENCE scheduler (config 5 geometry).

    REF_ROOT=/path/to/llm-inference-scheduler python tests/golden/make_golden_e2e.py

Builds the reference's own Qwen2Model (mini_engine/model/qwen2.py) on the CPU
in fp32 with the seeded random weights of pagedkv.model.random_weights, its
BlockManager and Scheduler (mini_engine/scheduler.py) with a stub tokenizer
whose EOS ids never occur, and runs the scenarios of
tests/golden/cases.py:e2e_scenarios to completion.  Writes the generated token
ids and the scheduler metrics to tests/golden/e2e_greedy.json.
"""

import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "llm-inference-scheduler_b200"))
import cases as C  # noqa: E402
from pagedkv.model import Qwen2Config, random_weights  # noqa: E402

sys.path.insert(0, os.environ.get("REF_ROOT", "/root/reference"))
from mini_engine.model.config import Qwen2Config as RefConfig  # noqa: E402
from mini_engine.model.qwen2 import Qwen2Model  # noqa: E402
from mini_engine.paged.block_manager import BlockManager  # noqa: E402
from mini_engine.sampling import SamplingParams  # noqa: E402
from mini_engine.scheduler import Request, Scheduler  # noqa: E402


class StubTokenizer:
    eos_ids = {-1}  # never produced


def run(model, sc):
    mgr = BlockManager(sc["num_blocks"], 16, 24, 2, 64, dtype=torch.float32)
    sched = Scheduler(model, StubTokenizer(), mgr, max_num_seqs=sc["max_num_seqs"],
                      max_batched_tokens=sc["max_batched_tokens"],
                      enable_prefix_cache=sc["prefix_cache"])
    reqs = []
    for i, p in enumerate(sc["prompts"]):
        r = Request(req_id=i, prompt_ids=list(p),
                    params=SamplingParams(temperature=0.0, max_new_tokens=sc["max_new_tokens"]))
        sched.waiting.append(r)
        reqs.append(r)
    while sched.has_work:
        sched.step()
    if sc["turn2_extra"] is not None:
        p = reqs[0].prompt_ids + reqs[0].output_ids + sc["turn2_extra"]
        r = Request(req_id=len(reqs), prompt_ids=p,
                    params=SamplingParams(temperature=0.0, max_new_tokens=sc["max_new_tokens"]))
        sched.waiting.append(r)
        reqs.append(r)
        while sched.has_work:
            sched.step()
    return dict(outputs=[r.output_ids for r in reqs], metrics=dict(sched.metrics),
                num_prefix_cached=[r.num_prefix_cached for r in reqs],
                preemptions=[r.preemptions for r in reqs])


def main():
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    cfg = Qwen2Config()
    t0 = time.time()
    w = random_weights(cfg, seed=C.E2E_SEED, final_norm_scale=C.E2E_FINAL_NORM_SCALE)
    model = Qwen2Model(RefConfig(), w)
    out = {"seed": C.E2E_SEED, "final_norm_scale": C.E2E_FINAL_NORM_SCALE}
    for name, sc in C.e2e_scenarios().items():
        out[name] = run(model, sc)
        print(name, out[name]["metrics"], f"{time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "e2e_greedy.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
