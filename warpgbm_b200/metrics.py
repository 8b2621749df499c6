"""Evaluation metrics of the reference (warpgbm/metrics.py:5-37), restated as
torch device ops so eval / early stopping decide exactly as the reference."""
import torch


def rmsle_torch(y_true, y_pred, eps=1e-7):
    y_true = torch.clamp(y_true, min=0)
    y_pred = torch.clamp(y_pred, min=0)
    return torch.sqrt(torch.mean((torch.log1p(y_true + eps) - torch.log1p(y_pred + eps)) ** 2))


def softmax(logits, dim=-1):
    """exp(x - max) / sum(exp(x - max)) as in metrics.py:12-15."""
    e = torch.exp(logits - torch.max(logits, dim=dim, keepdim=True)[0])
    return e / torch.sum(e, dim=dim, keepdim=True)


def log_loss_torch(y_true_labels, y_pred_probs, eps=1e-15):
    p = torch.clamp(y_pred_probs, eps, 1 - eps)
    n = y_true_labels.shape[0]
    return -torch.mean(torch.log(p[torch.arange(n, device=p.device), y_true_labels.long()]))


def accuracy_torch(y_true_labels, y_pred_labels):
    return (y_true_labels == y_pred_labels).float().mean()
