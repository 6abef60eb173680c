from .rfdetr import RFDETR, build_model
