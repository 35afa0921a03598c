"""HTTP serving (python/kinetic_rt/serve.py of the reference) is outside this
build's hot path; `serve` exists so the package's public names import."""


def serve(port=8000):
    raise NotImplementedError("the HTTP server is outside this build's decoder hot path")
