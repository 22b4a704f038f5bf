"""Golden greedy token streams of the REFERENCE scheduler run in fp16.

    REF_ROOT=/path/to/llm-inference-scheduler python tests/golden/make_golden_e2e_f16.py

The same scenarios and seeded weights as make_golden_e2e.py, but the
reference's own Qwen2Model (mini_engine/model/qwen2.py), BlockManager and
Scheduler (mini_engine/scheduler.py) run with fp16 weights and fp16 KV pools
on the CPU: the reference's fp16 rounding points (fp16 scores, fp32 softmax,
probabilities cast back to fp16, qwen2.py:98-128) are in the stream.

For every generated token it also records, from the row the token was
sampled from, the reference's top-2 token ids and their fp16 logits (so its
own margin, top-1 minus top-2).  A model wrapper (the scheduler sees only
.device and .forward) keeps each forward's per-sequence top-2, and the driver
assigns them to the requests that gained a token in that step.  A test that
feeds the same tokens to another implementation can then compare its logit
gap between the same two tokens with the reference's, token by token.
Writes tests/golden/e2e_greedy_f16.json.
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


class TopTwoRecorder:
    """The reference model, plus the top-2 (id, logit) pairs of every row."""

    def __init__(self, model):
        self.model = model
        self.device = model.device
        self.last: dict[int, tuple] = {}

    def forward(self, input_ids, seq_infos, kv_cache):
        logits = self.model.forward(input_ids, seq_infos, kv_cache)
        lf = logits.float()
        first = torch.argmax(lf, dim=-1)  # the greedy token (sampling.py: argmax)
        rest = lf.clone()
        rest[torch.arange(len(seq_infos)), first] = float("-inf")
        second = torch.argmax(rest, dim=-1)
        self.last = {s.seq_id: (int(first[i]), float(lf[i, first[i]]), int(second[i]),
                                float(lf[i, second[i]])) for i, s in enumerate(seq_infos)}
        return logits


def run(model, sc):
    mgr = BlockManager(sc["num_blocks"], 16, 24, 2, 64, dtype=torch.float16)
    rec = TopTwoRecorder(model)
    sched = Scheduler(rec, StubTokenizer(), mgr, max_num_seqs=sc["max_num_seqs"],
                      max_batched_tokens=sc["max_batched_tokens"],
                      enable_prefix_cache=sc["prefix_cache"])
    reqs, top2 = [], {}

    def drive():
        while sched.has_work:
            before = {r.req_id: len(r.output_ids) for r in reqs}
            sched.step()
            for r in reqs:
                if len(r.output_ids) > before[r.req_id]:
                    top2[r.req_id].append(rec.last[r.req_id])

    def submit(prompt):
        r = Request(req_id=len(reqs), prompt_ids=list(prompt),
                    params=SamplingParams(temperature=0.0, max_new_tokens=sc["max_new_tokens"]))
        sched.waiting.append(r)
        reqs.append(r)
        top2[r.req_id] = []

    for p in sc["prompts"]:
        submit(p)
    drive()
    if sc["turn2_extra"] is not None:
        submit(reqs[0].prompt_ids + reqs[0].output_ids + sc["turn2_extra"])
        drive()
    assert all(len(top2[r.req_id]) == len(r.output_ids) for r in reqs)
    # greedy = argmax: the sampled token is the top-1 id (first index on ties)
    assert all(t[0] == tok for r in reqs for t, tok in zip(top2[r.req_id], r.output_ids))
    return dict(outputs=[r.output_ids for r in reqs], metrics=dict(sched.metrics),
                margins=[[t[1] - t[3] for t in top2[r.req_id]] for r in reqs],
                top2=[[list(t) for t in top2[r.req_id]] for r in reqs],
                num_prefix_cached=[r.num_prefix_cached for r in reqs],
                preemptions=[r.preemptions for r in reqs])


def main():
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    cfg = Qwen2Config()
    t0 = time.time()
    w = random_weights(cfg, seed=C.E2E_SEED, final_norm_scale=C.E2E_FINAL_NORM_SCALE)
    model = Qwen2Model(RefConfig(), {k: v.half() for k, v in w.items()})
    out = {"seed": C.E2E_SEED, "final_norm_scale": C.E2E_FINAL_NORM_SCALE, "dtype": "float16",
           "torch": torch.__version__}
    for name, sc in C.e2e_scenarios().items():
        out[name] = run(model, sc)
        print(name, out[name]["metrics"], f"{time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "e2e_greedy_f16.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
