"""KernelCommandEncoder / KernelLibrary / scratch protocol on the GPU:
hazard tracking (KernelCommandEncoder.swift:155-168), library cache and
unknown names (Internals/KernelLibraryTests.swift), scratch borrow/release
(KernelCommandEncoder.swift:87-141), dispatch hook, graph capture."""
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


@pytest.fixture(scope="module")
def lib(pc):
    return pc.KernelLibrary(0)


def test_library_caches_pipeline_states(pc, lib):
    assert lib.pipeline_state("add") == lib.pipeline_state("add")
    assert "flash_decoding_partial_bf16" in lib.function_names


def test_library_unknown_function(pc, lib):
    with pytest.raises(pc.PopcornError) as e:
        lib.pipeline_state("does_not_exist")
    assert e.value == pc.PopcornError(pc.PopcornError.kernelFunctionNotFound, "")


def test_hazard_barriers(pc, lib):
    enc = pc.KernelCommandEncoder(lib)
    a, b, c, d, e = (torch.rand(64, device="cuda") for _ in range(5))
    K = pc.Kernels
    enc.encode(K.Add(a, b, into=c), K.Add(a, b, into=d))      # read/read, distinct writes
    assert enc.barrier_count == 0
    enc.encode(K.Add(c, b, into=e))                           # RAW on c
    assert enc.barrier_count == 1
    enc.encode(K.Add(d, d, into=a))                           # WAR on a? map was cleared: only e,c,b known
    assert enc.barrier_count == 1
    enc.encode(K.Mul(a, b, into=c))                           # RAW on a
    assert enc.barrier_count == 2
    enc.barrier()
    assert enc.barrier_count == 3
    enc.encode(K.Add(a, b, into=c), K.Add(d, e, into=c))      # WAW on c
    assert enc.barrier_count == 4
    torch.cuda.synchronize()
    assert torch.allclose(c, d + e)
    assert enc.dispatch_count == 7


def test_scratch_protocol_and_reuse(pc, lib):
    pool = pc.ScratchPool()
    enc = pc.KernelCommandEncoder(lib, scratch=pool)
    q = torch.randn(1, 8, 1, 256, device="cuda", dtype=torch.float16)
    k = torch.randn(1, 4, 1024, 256, device="cuda", dtype=torch.float16)
    out = torch.empty_like(q)
    fa = pc.Kernels.FlashAttention(q, k, k, into=out, scale=1 / 16)
    enc.encode(fa)
    assert pool.borrows == 3 and pool.reuses == 0 and not pool._live
    enc.encode(fa)
    assert pool.borrows == 6 and pool.reuses == 3
    torch.cuda.synchronize()


def test_scratch_failure_surfaces(pc, lib):
    class Broken(pc.KernelScratchAllocator):
        def borrow(self, length):
            raise pc.PopcornError(pc.PopcornError.workspaceExhausted, "no room")

    enc = pc.KernelCommandEncoder(lib, scratch=Broken())
    q = torch.randn(1, 8, 1, 256, device="cuda", dtype=torch.float16)
    k = torch.randn(1, 4, 1024, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(pc.PopcornError) as e:
        enc.encode(pc.Kernels.FlashAttention(q, k, k, into=torch.empty_like(q), scale=1 / 16))
    assert e.value.code == pc.PopcornError.workspaceExhausted
    assert enc.dispatch_count == 0
    enc2 = pc.KernelCommandEncoder(lib)  # no allocator at all
    with pytest.raises(pc.PopcornError) as e:
        enc2.encode(pc.Kernels.FlashAttention(q, k, k, into=torch.empty_like(q), scale=1 / 16))
    assert e.value.code == pc.PopcornError.tensorAllocationFailed


def test_dispatch_hook(pc, lib):
    enc = pc.KernelCommandEncoder(lib, scratch=pc.ScratchPool())
    seen = []
    enc.set_dispatch_hook(lambda name, phase, s: seen.append((name, phase)))
    q = torch.randn(1, 8, 1, 256, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 4, 4096, 256, device="cuda", dtype=torch.bfloat16)
    enc.encode(pc.Kernels.FlashAttention(q, k, k, into=torch.empty_like(q), scale=1 / 16))
    names = [n for n, p in seen if p == 0]
    assert names == ["flash_decoding_partial_bf16", "flash_decoding_reduce_bf16"]
    assert [p for _, p in seen] == [0, 1, 0, 1]
    torch.cuda.synchronize()


def test_graph_capture_replays(pc, lib):
    """A captured step replays with new device-side inputs."""
    enc_stream = torch.cuda.Stream()
    a = torch.rand(1000, device="cuda")
    b = torch.rand(1000, device="cuda")
    c = torch.empty_like(a)
    with torch.cuda.stream(enc_stream):
        enc = pc.KernelCommandEncoder(lib, stream=enc_stream)
        kern = pc.Kernels.Add(a, b, into=c)
        enc.encode(kern)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=enc_stream):
            enc.encode(kern)
        a.fill_(2.0)
        b.fill_(3.0)
        g.replay()
    torch.cuda.synchronize()
    assert torch.all(c == 5.0)
