"""Run by test_gpu_multi.py under torch.distributed.run with two ranks (one GPU
each): the sharded FramePipeline, whose next frame's decode and all-gather run
ahead of the current render, must give the images of frames rendered one at a
time with the exchange in line. Exits non-zero on any difference."""
import os, sys, torch, torch.distributed as dist
from datetime import timedelta
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "nest-splatting_b200"), os.path.join(HERE, ".."), HERE]
from helpers import small_scene
from nest_b200.frame import FrameRenderer, FramePipeline
from nest_b200.views import DecodeShard, shard_range
from nest_b200.camera import orbit_camera
from nest_b200 import raster
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
shard = DecodeShard.create(fr.rvq_idx, fr.dims, world, rank)
pipe = FramePipeline(fr, shard)
pipe.run(n, cams[0], lambda i: host_idx[i % 2], lambda i: host_cam[i % 2], lambda i: host_rgb[i])
torch.cuda.synchronize()
ok = True
lo, hi = shard_range(shard.P, world, rank)
for i in range(n):
    shard.idx_shard[: hi - lo].copy_(streams[i % 2][lo:hi].cuda())
    fr.decoded = shard.decode_and_gather(fr.codebooks, raster.rvq_decode)
    ref = fr.render(cams[i % 2], skip_decode=True).cpu()
    same = torch.equal(ref, host_rgb[i])
    ok &= same
    print(rank, i, same, float(ref.abs().sum()), flush=True)
dist.barrier()
dist.destroy_process_group()
sys.exit(0 if ok else 1)
