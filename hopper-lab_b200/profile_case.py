"""One GEMM launch inside cudaProfilerStart/Stop, for ncu captures.

  python hopper-lab_b200/profile_case.py <f16|e4m3> <ours|cublas> [variant] [size]

size: S (M = N = K = S), MxK (N = M) or MxNxK.

Three warm-up launches run first; ncu with --profile-from-start off then captures
only the fourth. 'cublas' runs torch.matmul (fp16) or torch._scaled_mm (e4m3) on
the same inputs as the reference column.
"""
import sys, torch, importlib.util
sys.path.insert(0, '.')
import __graft_entry__ as g
b200 = g._load_pkg()
dt, who = sys.argv[1], sys.argv[2]
variant = sys.argv[3] if len(sys.argv) > 3 else 'auto'
size = sys.argv[4] if len(sys.argv) > 4 else "8192"
if "x" in size:  # MxK (N = M) or MxNxK
    dims = [int(v) for v in size.split("x")]
    M, N, K = (dims[0], dims[0], dims[1]) if len(dims) == 2 else dims
else:
    M = N = K = int(size)
torch.cuda.set_device(0)
g_ = torch.Generator(device='cuda'); g_.manual_seed(0)
if dt == 'f16':
    a = (torch.rand((M, K), generator=g_, device='cuda') * 2 - 1).half()
    b = (torch.rand((N, K), generator=g_, device='cuda') * 2 - 1).half()
    c = torch.empty((M, N), dtype=torch.float16, device='cuda')
    sa = sb = None
else:
    qa, sa = b200.quantize_e4m3((torch.rand((M, K), generator=g_, device='cuda') * 2 - 1).contiguous())
    qb, sb = b200.quantize_e4m3((torch.rand((N, K), generator=g_, device='cuda') * 2 - 1).contiguous())
    a, b = qa.view(M, K), qb.view(N, K)
    c = torch.empty((M, N), dtype=torch.bfloat16, device='cuda')
def run():
    if who == 'ours':
        b200.gemm(a, b, c, scale_a=sa, scale_b=sb, variant=variant)
    elif dt == 'f16':
        torch.matmul(a, b.t(), out=c)
    else:
        torch._scaled_mm(a, b.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
for _ in range(3): run()
torch.cuda.synchronize()
torch.cuda.profiler.start()
run()
torch.cuda.synchronize()
torch.cuda.profiler.stop()
rc, bits = b200.status()
assert rc == 0, hex(bits)
print('ok', dt, who, variant)
