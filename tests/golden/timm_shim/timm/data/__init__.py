IMAGENET_DEFAULT_MEAN = (0.485, 0.456, 0.406)
IMAGENET_DEFAULT_STD = (0.229, 0.224, 0.225)


class AugMixDataset:  # placeholder
    pass


def create_dataset(*args, **kwargs):
    raise NotImplementedError("placeholder")


def create_loader(*args, **kwargs):
    raise NotImplementedError("placeholder")
