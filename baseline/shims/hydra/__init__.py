def main(*args, **kwargs):
    def deco(fn):
        return fn

    return deco
