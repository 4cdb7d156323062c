// ep.cu — expert parallelism for the prefill MoE block through the C ABI, over NCCL
// (moearc_x_ep_*; the exchange the Python driver moearc_b200/ep.py runs over torch.distributed).
//
// Each rank owns n_expert / n_ranks experts (loaded into its moearc_x_prefill object, whose
// route order is owner-major: rank r's experts are positions r * n_local .. (r + 1) * n_local - 1,
// moearc_x_prefill_set_order). One forward:
//   route      the rank's tokens, grouped by position (buffer 3: rows per position)
//   all-gather every rank's per-position counts (ncclAllGather, device to device)
//   plan       on the host: rows to send to / receive from each rank, and the received rows as
//              (source, local expert) segments — the one host synchronisation of the block, since
//              NCCL's point-to-point sizes are host arguments
//   dispatch   ncclSend / ncclRecv in one group: each rank's rows for rank r are one contiguous run
//              of its route buffer (positions are owner-major), received source-major
//   experts    the grouped GEMMs over the received segments
//   return     the result rows back in one group, to where the route step put each row
//   combine    per token, router order, plus the residual
// Everything after the plan is enqueued on the context stream without waiting. The NCCL functions
// are resolved at run time from the process (a host that already loaded NCCL and built the
// communicator) or from libnccl.so.2, so the library does not link NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

using namespace moearc;

namespace {

struct nccl_api {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    bool ok = false;
};

// The process's NCCL if one is loaded with global symbols, else libnccl.so.2.
const nccl_api &nccl() {
    static nccl_api api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = RTLD_DEFAULT;
        if (!dlsym(h, "ncclSend")) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto get = [&](const char *n) { return dlsym(h, n); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(get("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(get("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(get("ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(get("ncclAllGather"));
        api.send = reinterpret_cast<decltype(api.send)>(get("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(get("ncclRecv"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(get("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(get("ncclGroupEnd"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.send &&
                 api.recv && api.group_start && api.group_end;
    });
    return api;
}

}  // namespace

namespace moearc {
// For the batched decoder's expert-parallel step (batch.cu): an all-gather of `bytes` from every
// rank, and a grouped exchange in which block r of send (bytes, at send + r * send_stride) goes
// to rank r and block r of recv comes from rank r. Both only enqueue on s (capturable in a CUDA
// graph); ERR when NCCL is missing or a call fails.
int ep_all_gather(void *comm, const void *send, void *recv, size_t bytes, cudaStream_t s) {
    const nccl_api &n = nccl();
    if (!n.ok || !comm) return ERR;
    return n.all_gather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(comm), s) == ncclSuccess ? OK : ERR;
}

int ep_exchange(void *comm, int world, const void *send, size_t send_stride, void *recv, size_t recv_stride,
                size_t bytes, cudaStream_t s) {
    const nccl_api &n = nccl();
    if (!n.ok || !comm) return ERR;
    ncclComm_t cm = static_cast<ncclComm_t>(comm);
    if (n.group_start() != ncclSuccess) return ERR;
    bool ok = true;
    for (int r = 0; r < world; ++r) {
        ok &= n.send(static_cast<const uint8_t *>(send) + r * send_stride, bytes, ncclUint8, r, cm, s) == ncclSuccess;
        ok &= n.recv(static_cast<uint8_t *>(recv) + r * recv_stride, bytes, ncclUint8, r, cm, s) == ncclSuccess;
    }
    return (n.group_end() == ncclSuccess && ok) ? OK : ERR;
}
}  // namespace moearc

struct moearc_x_ep {
    moearc_ctx *c;
    moearc_x_prefill *p;
    ncclComm_t comm;
    int rank, world, H, I, E, K, n_local;
    unsigned max_rows, max_tokens;
    void *mem = nullptr;
    int *counts_all = nullptr;        // device [world][E]
    int *counts_host = nullptr;       // pinned copy
    uint16_t *recv = nullptr;         // [max_rows][H] bf16
    uint16_t *act = nullptr;          // [max_rows][I] bf16
    float *y = nullptr;               // [max_rows][H]
    float *y_back = nullptr;          // [max_tokens * K][H]
    std::vector<int> send, recvn, seg_counts, seg_expert;
    unsigned n_recv = 0;
};

extern "C" {

int moearc_x_ep_unique_id(void *id) {
    const nccl_api &n = nccl();
    if (!n.ok || !id) return ERR;
    ncclUniqueId u;
    if (n.get_unique_id(&u) != ncclSuccess) return ERR;
    std::memcpy(id, &u, sizeof(u));
    return OK;
}

int moearc_x_ep_comm_init(moearc_ctx *c, void **comm, int n_ranks, const void *id, int rank) {
    const nccl_api &n = nccl();
    if (!n.ok || !c || !comm || !id || n_ranks < 1 || rank < 0 || rank >= n_ranks) return ERR;
    if (cudaSetDevice(c->device) != cudaSuccess) return ERR;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclComm_t cm = nullptr;
    if (n.comm_init_rank(&cm, n_ranks, u, rank) != ncclSuccess) return ERR;
    *comm = cm;
    return OK;
}

int moearc_x_ep_comm_destroy(void *comm) {
    const nccl_api &n = nccl();
    if (!n.ok || !comm) return ERR;
    return n.comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? OK : ERR;
}

moearc_x_ep *moearc_x_ep_create(moearc_ctx *c, moearc_x_prefill *p, const moearc_x_moe_desc *d, void *comm, int rank,
                               int n_ranks, unsigned max_rows) {
    if (!c || !p || !d || !comm || n_ranks < 1 || rank < 0 || rank >= n_ranks || d->n_expert % n_ranks) return nullptr;
    if (!nccl().ok) return nullptr;
    auto *ep = new moearc_x_ep();
    ep->c = c;
    ep->p = p;
    ep->comm = static_cast<ncclComm_t>(comm);
    ep->rank = rank;
    ep->world = n_ranks;
    ep->H = (int)d->n_embd;
    ep->I = (int)d->n_ff;
    ep->E = (int)d->n_expert;
    ep->K = (int)d->k;
    ep->n_local = ep->E / n_ranks;
    ep->max_rows = max_rows;
    ep->max_tokens = d->max_tokens;
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t b_cnt = up(sizeof(int) * (size_t)n_ranks * ep->E);
    const size_t b_recv = up((size_t)max_rows * ep->H * 2), b_act = up((size_t)max_rows * ep->I * 2);
    const size_t b_y = up(sizeof(float) * (size_t)max_rows * ep->H);
    const size_t b_back = up(sizeof(float) * (size_t)ep->max_tokens * ep->K * ep->H);
    if (cudaMalloc(&ep->mem, b_cnt + b_recv + b_act + b_y + b_back) != cudaSuccess ||
        cudaMallocHost(&ep->counts_host, sizeof(int) * (size_t)n_ranks * ep->E) != cudaSuccess) {
        cudaGetLastError();
        if (ep->mem) cudaFree(ep->mem);
        delete ep;
        return nullptr;
    }
    uint8_t *b = static_cast<uint8_t *>(ep->mem);
    ep->counts_all = reinterpret_cast<int *>(b);
    ep->recv = reinterpret_cast<uint16_t *>(b + b_cnt);
    ep->act = reinterpret_cast<uint16_t *>(b + b_cnt + b_recv);
    ep->y = reinterpret_cast<float *>(b + b_cnt + b_recv + b_act);
    ep->y_back = reinterpret_cast<float *>(b + b_cnt + b_recv + b_act + b_y);
    return ep;
}

void moearc_x_ep_destroy(moearc_x_ep *ep) {
    if (!ep) return;
    cudaStreamSynchronize(ep->c->stream);
    cudaFree(ep->mem);
    cudaFreeHost(ep->counts_host);
    delete ep;
}

int moearc_x_ep_forward(moearc_x_ep *ep, const unsigned short *x, unsigned n_tokens, const float *router_w,
                        const float *router_b, const float *residual, float *out) {
    if (!ep || !x || !router_w || !out) return ERR;
    if (n_tokens > ep->max_tokens) return ERR_ARG;
    const nccl_api &n = nccl();
    cudaStream_t s = ep->c->stream;
    const int W = ep->world, E = ep->E, nl = ep->n_local, H = ep->H;
    int rc = moearc_x_prefill_route(ep->p, x, n_tokens, router_w, router_b);
    if (rc) return rc;
    // every rank's per-position counts, then the plan on the host
    const int *cnt = static_cast<const int *>(moearc_x_prefill_buffer(ep->p, 3));
    if (n.all_gather(cnt, ep->counts_all, (size_t)E, ncclInt32, ep->comm, s) != ncclSuccess) return ERR;
    if (cudaMemcpyAsync(ep->counts_host, ep->counts_all, sizeof(int) * (size_t)W * E, cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return ERR;
    const int *ca = ep->counts_host;
    const int lo = ep->rank * nl;
    ep->send.assign(W, 0);
    ep->recvn.assign(W, 0);
    ep->seg_counts.resize((size_t)W * nl);
    ep->seg_expert.resize((size_t)W * nl);
    for (int r = 0; r < W; ++r)
        for (int j = 0; j < nl; ++j) {
            ep->send[r] += ca[(size_t)ep->rank * E + r * nl + j];
            const int c_in = ca[(size_t)r * E + lo + j];
            ep->recvn[r] += c_in;
            ep->seg_counts[(size_t)r * nl + j] = c_in;
            ep->seg_expert[(size_t)r * nl + j] = j;
        }
    unsigned n_recv = 0;
    for (int r = 0; r < W; ++r) n_recv += (unsigned)ep->recvn[r];
    if (n_recv > ep->max_rows) return ERR_ARG;
    ep->n_recv = n_recv;
    // dispatch: this rank's rows for rank r are one run of the route buffer; received source-major
    const uint16_t *xp = static_cast<const uint16_t *>(moearc_x_prefill_buffer(ep->p, 6));
    const size_t row16 = (size_t)H * 2;
    if (n.group_start() != ncclSuccess) return ERR;
    size_t so = 0, ro = 0;
    bool ok = true;
    for (int r = 0; r < W; ++r) {
        if (ep->send[r]) ok &= n.send(xp + so * H, (size_t)ep->send[r] * row16, ncclUint8, r, ep->comm, s) == ncclSuccess;
        if (ep->recvn[r])
            ok &= n.recv(ep->recv + ro * H, (size_t)ep->recvn[r] * row16, ncclUint8, r, ep->comm, s) == ncclSuccess;
        so += (size_t)ep->send[r];
        ro += (size_t)ep->recvn[r];
    }
    if (n.group_end() != ncclSuccess || !ok) return ERR;
    if (n_recv) {
        rc = moearc_x_prefill_experts(ep->p, ep->recv, n_recv, ep->seg_counts.data(), ep->seg_expert.data(),
                                      (unsigned)ep->seg_counts.size(), ep->act, ep->y);
        if (rc) return rc;
    }
    // the result rows home, to where the route step put each row
    if (n.group_start() != ncclSuccess) return ERR;
    so = ro = 0;
    for (int r = 0; r < W; ++r) {
        if (ep->recvn[r]) ok &= n.send(ep->y + ro * H, (size_t)ep->recvn[r] * H, ncclFloat32, r, ep->comm, s) == ncclSuccess;
        if (ep->send[r])
            ok &= n.recv(ep->y_back + so * H, (size_t)ep->send[r] * H, ncclFloat32, r, ep->comm, s) == ncclSuccess;
        so += (size_t)ep->send[r];
        ro += (size_t)ep->recvn[r];
    }
    if (n.group_end() != ncclSuccess || !ok) return ERR;
    return moearc_x_prefill_combine(ep->p, ep->y_back, n_tokens, residual, out);
}

int moearc_x_ep_counts(moearc_x_ep *ep, int *counts_all) {
    if (!ep || !counts_all) return ERR;
    std::memcpy(counts_all, ep->counts_host, sizeof(int) * (size_t)ep->world * ep->E);
    return OK;
}

unsigned moearc_x_ep_received(moearc_x_ep *ep) { return ep ? ep->n_recv : 0u; }

}  // extern "C"
