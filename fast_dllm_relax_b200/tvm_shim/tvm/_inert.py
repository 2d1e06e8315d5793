"""Attribute sink for TVM graph-construction helpers that the runtime never calls."""


class _Inert:
    def __init__(self, path: str):
        self._path = path

    def __getattr__(self, item):
        if item.startswith("__"):
            raise AttributeError(item)
        return _Inert(f"{self._path}.{item}")

    def __call__(self, *args, **kwargs):
        raise NotImplementedError(
            f"{self._path} is not available: no Relax graph is built against the sm_100a library")
