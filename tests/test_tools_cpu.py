"""HF conversion, loss comparison and generation utilities on CPU."""
import os

import pytest
import torch


def test_hf_conversion_round_trip(tmp_path):
    from safetensors.torch import load_file, save_file

    from torchtitan_b200.checkpoint_conversion import convert_from_hf, convert_to_hf
    from torchtitan_b200.models.llama3 import model_registry

    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    model = spec.model.build()
    model.init_weights()
    hf = spec.state_dict_adapter(spec.model, None).to_hf({k: v.detach() for k, v in model.state_dict().items()})
    hf_dir = tmp_path / "hf"
    hf_dir.mkdir()
    save_file({k: v.contiguous() for k, v in hf.items()}, str(hf_dir / "model.safetensors"))
    state = convert_from_hf(str(hf_dir), str(tmp_path / "dcp"), "llama3", "debugmodel")
    for k, v in model.state_dict().items():
        assert torch.equal(state[k], v), k
    convert_to_hf(str(tmp_path / "dcp"), str(tmp_path / "hf_out"), "llama3", "debugmodel", "float32")
    back = load_file(str(tmp_path / "hf_out" / "model.safetensors"))
    assert set(back) == set(hf)
    for k in hf:
        assert torch.equal(back[k], hf[k]), k
    assert os.path.exists(tmp_path / "hf_out" / "model.safetensors.index.json")


def test_loss_compare_detects_differences(tmp_path):
    from torchtitan_b200.loss_compare import compare, main

    assert compare({1: 1.0, 2: 0.5}, {1: 1.0, 2: 0.5}, True, 0.0) == []
    assert len(compare({1: 1.0, 2: 0.5}, {1: 1.0, 2: 0.50001}, True, 0.0)) == 1
    assert compare({1: 1.0}, {1: 1.00001}, False, 1e-4) == []
    opts = ("--training.seq-len 64 --training.local-batch-size 2 --training.dtype float32 "
            "--training.mixed-precision-param float32 --activation-checkpoint.mode none")
    common = [".", ".", "--baseline-config", "llama3_debugmodel", "--steps", "3", "--baseline-options", opts]
    exp = tmp_path / "losses.txt"
    rc = main(common + ["--test-options", opts, "--assert-equal", "--output-folder", str(tmp_path / "a"),
                        "--export-result", str(exp)])
    assert rc == 0 and len(exp.read_text().splitlines()) == 3
    assert (tmp_path / "a" / "seed" / "checkpoint" / "step-0" / ".metadata").exists()
    rc = main(common + ["--test-options", opts + " --optimizer.lr 1e-2", "--assert-equal", "--output-folder",
                        str(tmp_path / "b")])
    assert rc == 1
    # recorded curve: the baseline alone must reproduce it
    assert main(common + ["--baseline-only", "--import-result", str(exp), "--assert-equal"]) == 0


def test_loss_compare_seed_checkpoint_across_layouts(tmp_path):
    """From one seed checkpoint, one process and two tensor-parallel ranks (gloo, same data on
    both) give the same curve within fp32 reduction-order tolerance."""
    from torchtitan_b200.loss_compare import main

    opts = ("--training.seq-len 64 --training.local-batch-size 2 --training.dtype float32 "
            "--training.mixed-precision-param float32 --activation-checkpoint.mode none")
    rc = main([".", ".", "--baseline-config", "llama3_debugmodel_cpu", "--steps", "3", "--baseline-options", opts,
               "--test-options", opts + " --parallelism.tensor-parallel-degree 2 "
               "--parallelism.data-parallel-shard-degree 1", "--test-ngpus", "2", "--rtol", "1e-4",
               "--output-folder", str(tmp_path)])
    assert rc == 0, (tmp_path / "summary.txt").read_text()


def test_seed_checkpoint_sets_initial_weights(tmp_path):
    """A seed checkpoint (model only, step 0) gives a run with another seed the same weights."""
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    args = ["--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
            "--training.dtype", "float32", "--training.mixed-precision-param", "float32", "--checkpoint.enable"]
    a = Trainer(ConfigManager().parse_args(args + ["--debug.seed", "1", "--dump-folder", str(tmp_path / "a")]))
    path = a.checkpointer.save_seed()
    wa = {k: v.detach().clone() for k, v in a.model_parts[0].state_dict().items()}
    a.close()
    b = Trainer(ConfigManager().parse_args(args + ["--debug.seed", "2", "--dump-folder", str(tmp_path / "b"),
                                                   "--checkpoint.initial-load-path", path]))
    wb = b.model_parts[0].state_dict()
    assert any(not torch.equal(wa[k], wb[k]) for k in wa)  # different seeds, different weights
    assert b.checkpointer.load()
    assert all(torch.equal(wa[k], b.model_parts[0].state_dict()[k]) for k in wa)
    b.close()


def test_generate_greedy_and_eos():
    from torchtitan_b200.generate import generate
    from torchtitan_b200.models.llama3 import model_registry

    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    model = spec.model.build()
    model.init_weights()
    model.eval()
    p = torch.tensor([[1, 2, 3]])
    a = generate(model, p, 5)
    b = generate(model, p, 5)
    assert a.shape == (1, 8) and torch.equal(a, b)
    assert int(a[0, 3]) == int(model(p)[0, -1].argmax())
    eos = int(a[0, 3])
    c = generate(model, p, 5, eos_id=eos)
    assert c.shape == (1, 4)
    g = torch.Generator().manual_seed(0)
    s = generate(model, p, 4, temperature=1.0, top_k=5, generator=g)
    assert s.shape == (1, 7)


def test_forge_engine_steps_on_given_batches(tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.forge import ForgeEngine

    cfg = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
                                      "--training.local-batch-size", "2", "--training.dtype", "float32",
                                      "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode",
                                      "none", "--dump-folder", str(tmp_path)])
    eng = ForgeEngine(cfg)
    tokens = torch.randint(0, 2048, (2, 65))
    batch = ({"input": tokens[:, :-1]}, tokens[:, 1:])
    l1 = float(eng.train_on_batches([batch]))
    for _ in range(4):
        l2 = float(eng.train_on_batches([batch]))
    assert eng.step == 5 and l2 < l1  # the same batch is being memorised
    assert eng.forward(batch[0]).shape == (2, 64, 2048)
    eng.close()


@pytest.mark.parametrize("module", ["llama3", "qwen3", "deepseek_v3"])
def test_kv_cache_generation_equals_full_recompute(module):
    """Incremental decoding with the KV cache gives the same tokens as re-running the whole
    sequence, greedy and sampled, and leaves no cache behind."""
    import importlib

    from torchtitan_b200.generate import _cache_layers, generate

    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry("debugmodel")
    torch.manual_seed(0)
    m = spec.model.build()
    m.init_weights()
    m.eval()
    atts = _cache_layers(m)
    assert atts is not None
    p = torch.randint(0, 2048, (2, 7))
    with torch.no_grad():
        assert torch.equal(generate(m, p, 6), generate(m, p, 6, use_cache=False))
        a = generate(m, p, 6, 1.0, 5, torch.Generator().manual_seed(1))
        b = generate(m, p, 6, 1.0, 5, torch.Generator().manual_seed(1), use_cache=False)
    assert torch.equal(a, b) and all(x.kv_cache is None for x in atts)


def test_forge_example_loop_matches_trainer(tmp_path):
    """The engine-driven loop reproduces the trainer's own loop on the same config."""
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.forge import ForgeEngine, example_train
    from torchtitan_b200.trainer import Trainer

    args = ["--module", "llama3", "--config", "llama3_debugmodel", "--training.seq-len", "64",
            "--training.local-batch-size", "2", "--training.dtype", "float32", "--training.steps", "3",
            "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
            "--debug.seed", "0"]
    eng = ForgeEngine(ConfigManager().parse_args(args + ["--dump-folder", str(tmp_path / "a")]))
    got = example_train(eng)
    eng.close()
    t = Trainer(ConfigManager().parse_args(args + ["--dump-folder", str(tmp_path / "b")]))
    want = []
    it = t.batch_generator(t.dataloader)
    while t.step < 3:
        t.step += 1
        want.append(float(t.train_step(it)))
    t.close()
    assert got == want and len(got) == 3


def test_loss_compare_checks_out_a_revision(tmp_path):
    """A git revision runs from its own temporary worktree, which is removed afterwards."""
    import subprocess

    from torchtitan_b200 import loss_compare

    r = subprocess.run(["git", "rev-parse", "--verify", "HEAD"], cwd=loss_compare.HERE, capture_output=True)
    if r.returncode:
        pytest.skip("not a git checkout")
    seen = []
    real = loss_compare._launch
    loss_compare._launch = lambda tree, args, n, log: (seen.append(tree), real(tree, args, n, log))[1]
    try:
        opts = ("--training.seq-len 32 --training.local-batch-size 1 --training.dtype float32 "
                "--training.mixed-precision-param float32 --activation-checkpoint.mode none")
        rc = loss_compare.main(["HEAD", ".", "--steps", "1", "--no-seed-checkpoint", "--baseline-options", opts,
                                "--test-options", opts, "--rtol", "1.0"])
    finally:
        loss_compare._launch = real
    assert rc == 0
    assert seen[0] != loss_compare.HERE and seen[1] == loss_compare.HERE
    assert not os.path.exists(seen[0])
    wt = subprocess.run(["git", "worktree", "list"], cwd=loss_compare.HERE, capture_output=True, text=True).stdout
    assert seen[0] not in wt
