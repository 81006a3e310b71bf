"""``jax.tree_util`` subset on torch for pytrees that are flat dicts of
arrays (fixture generation only): leaves in sorted-key order with
``DictKey`` paths, as JAX orders and names dict entries."""


class DictKey:
    def __init__(self, key):
        self.key = key

    def __repr__(self):
        return f"DictKey(key={self.key!r})"


class _Treedef:
    def __init__(self, keys):
        self.keys = keys

    def unflatten(self, leaves):
        return dict(zip(self.keys, leaves))


def tree_flatten_with_path(tree, is_leaf=None):
    keys = sorted(tree)
    return [((DictKey(k),), tree[k]) for k in keys], _Treedef(keys)


def tree_map(f, tree, *rest):
    return {k: f(tree[k], *(r[k] for r in rest)) for k in sorted(tree)}


def tree_map_with_path(f, tree, *rest):
    return {k: f((DictKey(k),), tree[k], *(r[k] for r in rest)) for k in sorted(tree)}
