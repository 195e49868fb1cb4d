/*
 * frame_order.h — where the frames of one video stream run when several GPUs share it, and when
 * they count as finished (host-only bookkeeping of ajib_video_multi, video_multi.cpp; no CUDA).
 *
 * Frame k of the stream (ticket k + 1) goes to device k mod n, into slot (k / n) mod depth of
 * that device's ring of frame buffers. A slot is reused only after its previous frame has
 * finished, so each device has at most `depth` frames in flight. Frames can finish out of order
 * across devices; the stream's completion is the longest prefix of finished tickets, so results
 * are handed back in submission order, the order a single-device player sees them (the
 * reference harness's one-stream loop, src/harness.c:646-700).
 */
#pragma once

#include <cstdint>
#include <vector>

namespace ajib {

class FrameOrder {
public:
    struct Place {
        int64_t ticket = 0;  // 1-based, in submission order
        int device = 0;      // index into the stream's device list
        int slot = 0;        // ring slot on that device
        int64_t reuse = 0;   // the slot's previous ticket, which must finish first (0: none)
    };

    FrameOrder(int ndev, int depth) : ndev_(ndev < 1 ? 1 : ndev), depth_(depth < 1 ? 1 : depth)
    {
        slot_ticket_.assign((size_t)ndev_ * depth_, 0);
    }

    int devices() const { return ndev_; }
    int depth() const { return depth_; }

    // The place of the next frame.
    Place next()
    {
        Place p;
        const int64_t k = next_ - 1;
        p.ticket = next_++;
        p.device = (int)(k % ndev_);
        p.slot = (int)((k / ndev_) % depth_);
        int64_t &occ = slot_ticket_[(size_t)p.device * depth_ + p.slot];
        p.reuse = occ;
        occ = p.ticket;
        if (p.ticket - done_base_ > (int64_t)done_.size()) done_.resize((size_t)(p.ticket - done_base_), 0);
        return p;
    }

    // Records that ticket t finished; returns the number of tickets finished in order (every
    // ticket up to it has finished).
    int64_t mark_done(int64_t t)
    {
        if (t > completed_ && t < next_) {
            done_[(size_t)(t - done_base_ - 1)] = 1;
            while (completed_ - done_base_ < (int64_t)done_.size() && done_[(size_t)(completed_ - done_base_)]) completed_++;
            // drop the finished prefix now and then, so the record stays as long as the frames in flight
            if (completed_ - done_base_ > 4096) {
                done_.erase(done_.begin(), done_.begin() + (completed_ - done_base_));
                done_base_ = completed_;
            }
        }
        return completed_;
    }

    bool finished(int64_t t) const
    {
        if (t <= completed_) return true;
        if (t >= next_) return false;
        return done_[(size_t)(t - done_base_ - 1)] != 0;
    }
    int64_t completed() const { return completed_; }
    int64_t issued() const { return next_ - 1; }

private:
    int ndev_, depth_;
    int64_t next_ = 1, completed_ = 0, done_base_ = 0;
    std::vector<int64_t> slot_ticket_;
    std::vector<uint8_t> done_;  // per ticket done_base_ + 1 + i
};

}  // namespace ajib
