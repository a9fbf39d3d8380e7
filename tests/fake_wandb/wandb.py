"""Stand-in for the wandb package in the metrics test: records init / log calls
to the JSON file named by HB_FAKE_WANDB_OUT."""
import json
import os

_calls = []


def _dump():
    with open(os.environ["HB_FAKE_WANDB_OUT"], "w") as f:
        json.dump(_calls, f)


class Table:
    def __init__(self, data=None, columns=None):
        self.data, self.columns = data, columns


class plot:  # noqa: N801 (mirrors wandb.plot)
    @staticmethod
    def bar(table, x, y, title=None):
        return {"bar": [x, y], "title": title, "rows": len(table.data)}


class _Run:
    def finish(self):
        _calls.append({"finish": True})
        _dump()


def init(**kw):
    _calls.append({"init": sorted(kw)})
    _dump()
    return _Run()


def log(d, step=None):
    _calls.append({"log": {k: (v if isinstance(v, (int, float, str, dict)) else str(v)) for k, v in d.items()},
                   "step": step})
    _dump()
