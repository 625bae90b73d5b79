"""Drop-in for the reference package of the same name (see the modules inside).

The package path is extended with every other directory of this name on
sys.path, so with ``PYTHONPATH=turbo-llm_b200:<reference checkout>`` the
modules defined here replace the reference's and the reference's other
modules of the package (e.g. ``execution.layer_executor``,
``cache.kv_cache``) still import from its checkout.
"""
from pkgutil import extend_path

__path__ = extend_path(__path__, __name__)
