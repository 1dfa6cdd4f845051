"""Run by test_gpu_multi.py under torch.distributed.run with two ranks (one GPU
each): the sharded FramePipeline (each rank decodes its surfel range, the
10 geometric attribute columns are all-gathered, the next frame's exchange runs
ahead of the current render) must give, bit for bit, the images of the same
frames rendered on one GPU alone from a full local decode. Exits non-zero on
any difference."""
import os, sys, torch, torch.distributed as dist
from datetime import timedelta
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "nest-splatting_b200"), os.path.join(HERE, ".."), HERE]
from helpers import small_scene
from nest_b200.frame import FrameRenderer, FramePipeline
from nest_b200.views import DecodeShard
from nest_b200.camera import orbit_camera
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
sc = small_scene(n=3000, seed=23, rvq=True)
fr = FrameRenderer(sc, device=f"cuda:{rank}")
W, H = sc.camera.width, sc.camera.height
cams = [orbit_camera(W, H, 50.0, 4.0, az + 90.0 * rank) for az in (0.0, 40.0)]
g = torch.Generator().manual_seed(5)
streams = [sc.rvq_idx.clone(), torch.randint(0, 256, sc.rvq_idx.shape, generator=g).to(torch.uint8)]
host_idx = [s.pin_memory() for s in streams]
host_cam = [torch.stack([c.world_view_transform, c.full_proj_transform]).contiguous().pin_memory() for c in cams]
n = 6
host_rgb = [torch.empty((3, H, W)).pin_memory() for _ in range(n)]
shard = DecodeShard.create(fr.rvq_idx, fr.dims, world, rank, columns=10)
pipe = FramePipeline(fr, shard)
pipe.run(n, cams[0], lambda i: host_idx[i % 2], lambda i: host_cam[i % 2], lambda i: host_rgb[i])
torch.cuda.synchronize()
ok = True
local = torch.empty((fr.P, fr.dims), dtype=torch.float32, device=fr.device)
for i in range(n):
    # the single-GPU frame: every row decoded on this GPU, no exchange
    fr.decoded = local
    ref = fr.render(cams[i % 2], rvq_idx=streams[i % 2].to(fr.device)).cpu()
    same = torch.equal(ref, host_rgb[i])
    ok &= same
    print(rank, i, same, float(ref.abs().sum()), flush=True)
dist.barrier()
dist.destroy_process_group()
sys.exit(0 if ok else 1)
