"""Stand-in for ``mlx.nn``: only ``Module`` is referenced (in annotations)."""


class Module:
    def children(self):
        return {}
