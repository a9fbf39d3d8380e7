"""Config files for the trainer (``--config_file``): YAML, TOML and JSON.

The reference configures runs only through argparse and shell presets
(train.py:171-226) and lists config files as future work (README.md:133).
"""
import json

import pytest

from heiretsu_b200.trainer import build_argparser, parse_args


def _write(tmp_path, name, text):
    p = tmp_path / name
    p.write_text(text)
    return str(p)


@pytest.mark.parametrize("name,text", [
    ("run.yaml", "n_layer: 12\nn_head: 12\nbetas: [0.8, 0.99]\nsynthetic_data: true\namp: bf16\ndp: 2\n"),
    ("run.toml", "n_layer = 12\nn_head = 12\nbetas = [0.8, 0.99]\nsynthetic_data = true\namp = \"bf16\"\ndp = 2\n"),
    ("run.json", json.dumps({"n_layer": 12, "n_head": 12, "betas": [0.8, 0.99], "synthetic_data": True,
                             "amp": "bf16", "dp": 2})),
])
def test_file_sets_defaults_and_command_line_wins(tmp_path, name, text):
    path = _write(tmp_path, name, text)
    a = parse_args(["--config_file", path, "--n_head", "16"])
    assert a.n_layer == 12 and a.n_head == 16 and a.dp == 2
    assert tuple(a.betas) == (0.8, 0.99)
    assert a.synthetic_data is True and a.amp == "bf16"
    assert a.n_embed == build_argparser().get_default("n_embed")  # untouched keys keep their defaults


def test_unknown_key_and_bad_choice_are_errors(tmp_path):
    with pytest.raises(ValueError, match="unknown keys"):
        parse_args(["--config_file", _write(tmp_path, "a.yaml", "n_layers: 3\n")])
    with pytest.raises(ValueError, match="not one of"):
        parse_args(["--config_file", _write(tmp_path, "b.yaml", "amp: fp8\n")])
    with pytest.raises(ValueError, match="expected 2 values"):
        parse_args(["--config_file", _write(tmp_path, "c.yaml", "betas: [0.9]\n")])
    with pytest.raises(ValueError, match="extension"):
        parse_args(["--config_file", _write(tmp_path, "d.ini", "x=1\n")])


@pytest.mark.parametrize("ext", ["yaml", "toml", "json"])
def test_save_config_round_trip(tmp_path, ext):
    out = str(tmp_path / f"resolved.{ext}")
    a = parse_args(["--n_layer", "7", "--dp", "2", "--betas", "0.85", "0.97", "--wandb", "--save_config", out])
    b = parse_args(["--config_file", out])
    va, vb = vars(a), vars(b)
    for k in va:
        if k in ("config_file", "save_config"):
            continue
        assert (tuple(va[k]) if isinstance(va[k], (list, tuple)) else va[k]) == \
            (tuple(vb[k]) if isinstance(vb[k], (list, tuple)) else vb[k]), k
