"""The reference's own CLI, `pickle infer`, end to end on the GPU.

oracle/_ref/pickle_cli_ref is the reference's unmodified ./pickle (its
src/pickle_cli.c, pickle_host.c, ... compiled from its sources);
oracle/_ref/pickle_cli_cuda is the same CLI built the way the PICKLE_CUDA=1
target of lestramanika_b200/hook/pickle_makefile_cuda.patch builds it:
src/pickle_fast.c with pickle_fast_cuda_hook.patch, the glue
pickle_cuda_hook.c and libpickle_cuda.so. Nothing else differs: the
unmodified pickle_chat_loop (src/pickle_host.c:410-535) tokenises the
prompt, prefills it and decodes greedily, and every attention block of
every token runs on the B200 through the shim.

North_star bar: greedy-decoded token ids identical to the unmodified build.
The tiny model's vocabulary maps every id to a distinct piece, so identical
generated text means identical ids."""
import os
import subprocess

import pytest

import oracle

pytestmark = pytest.mark.gpu

N_NEW = 200          # 17 prompt tokens + 200 fill 217 of the model's 256 positions


def _run(exe, model, env=None):
    if not os.path.exists(exe):
        pytest.fail(f"{exe} is not built (python -m lestramanika_b200.build --all --ref=...)")
    r = subprocess.run([exe, "infer", model, "hello world", str(N_NEW)], capture_output=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    text, _, stats = r.stdout.rpartition(b"\n--- ")
    return text, stats.decode(errors="replace"), r.stderr.decode(errors="replace")


@pytest.fixture(scope="module")
def vocab_model(tmp_path_factory):
    import make_tiny_llama
    path = str(tmp_path_factory.mktemp("cli") / "tiny_vocab.gguf")
    make_tiny_llama.write_model(path, 0, vocab=True)
    return path


def test_pickle_infer_on_the_gpu_matches_the_unmodified_cli(vocab_model):
    ref_text, ref_stats, _ = _run(os.path.join(oracle.REF_DIR, "pickle_cli_ref"), vocab_model)
    env = dict(os.environ, PICKLE_CUDA_VERBOSE="1", PICKLE_CUDA_DEVICE="0")
    gpu_text, gpu_stats, gpu_err = _run(os.path.join(oracle.REF_DIR, "pickle_cli_cuda"), vocab_model, env)
    assert "pickle_cuda: attention of 6 layers" in gpu_err, gpu_err      # the shim served the attention
    assert ref_stats.split(" in ")[0] == gpu_stats.split(" in ")[0]     # "17 prompt tokens, N generated"
    assert "17 prompt tokens" in ref_stats
    assert len(ref_text) > N_NEW
    assert gpu_text == ref_text
