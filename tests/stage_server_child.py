"""A stage server process for tests/test_gpu_stage_server.py: builds the
seeded synthetic model of the given config on GPU 0, serves its layers
through stage_server.StageServer, prints its port, and serves until
killed. With --fail-after N it drops a stage's connection on its N-th
forward (a simulated crash); --fail-from L limits that to the shard
starting at layer L."""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rakkan-mesh_b200"))

import rkcuda as rk  # noqa: E402
import stage_server as ss  # noqa: E402
import synth  # noqa: E402

p = argparse.ArgumentParser()
p.add_argument("--config", required=True)
p.add_argument("--seed", type=int, required=True)
p.add_argument("--fail-after", type=int, default=0)
p.add_argument("--fail-from", type=int, default=-1, help="only the shard starting at this layer fails")
args = p.parse_args()
over = json.loads(args.config)
c = synth.config("", over.pop("dtype", "q8_0"), **over)
dev = rk.Device(0)
dm = synth.DeviceModel(dev, c, args.seed)
count = {}


def fail_next(shard):
    count[shard] = count.get(shard, 0) + 1
    if args.fail_from >= 0 and shard[1] != args.fail_from:
        return False
    return args.fail_after > 0 and count[shard] == args.fail_after


srv = ss.StageServer(ss.cuda_stage_opener(dev, c, dm.layers), fail_next=fail_next)
print(srv.address[1], flush=True)
srv.serve_forever()
