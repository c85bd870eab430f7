"""Stand-in for the `easydict` package (absent from this image), which the reference engine's sampler imports for three
attribute-style dictionaries (prefilling_dllm_engine/prefilling_dllm/layers/sampler.py:9, 94-96). TEST INFRASTRUCTURE ONLY:
put on sys.path by oracle/build_ref.load_reference_engine() when the real package cannot be imported."""


class EasyDict(dict):
    """A dict whose keys also read and write as attributes, nested dicts included."""

    def __init__(self, data=None, **kwargs):
        super().__init__()
        for key, value in dict(data or {}, **kwargs).items():
            self[key] = value

    def __setitem__(self, key, value):
        if isinstance(value, dict) and not isinstance(value, EasyDict):
            value = EasyDict(value)
        super().__setitem__(key, value)

    def __getattr__(self, key):
        try:
            return self[key]
        except KeyError as exc:
            raise AttributeError(key) from exc

    def __setattr__(self, key, value):
        self[key] = value
