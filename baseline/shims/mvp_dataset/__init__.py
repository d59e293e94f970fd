"""Names the reference's kit modules import from mvp_dataset; unused by the reference arm."""


class Dataset:
    def __init__(self, *a, **k):
        raise RuntimeError("mvp_dataset is not available offline; the reference arm feeds synthetic packs")


class TorchLoader(Dataset):
    pass
